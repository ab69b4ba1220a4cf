"""The decoder step of oracle/model.py run sharded over torch.distributed ranks (gloo, CPU).
TEST INFRASTRUCTURE ONLY.

Each rank holds a trixium_b200.tp.TPWeights shard (the same rows, heads and segment order the GPU
engine uses) and computes its rows with the oracle's arithmetic; the all-gathers are gloo
collectives in rank order.  Its tokens must equal the unsharded OracleModel's: row sharding with
all-gathered inputs changes no arithmetic, so this pins the shard plan (row ranges, head
renumbering, grouped-output blocks, global argmax rows) on the CPU.
"""

import numpy as np
import torch
import torch.distributed as dist

from . import ref
from .model import Proj, _single

f32 = np.float32


def _segments(sp):
    """Proj per segment of a trixium_b200.tp.ShardPacked."""
    from trixium_b200 import layout as L
    data = sp.data.cpu().numpy()
    rb = L.row_bytes(sp.cols, sp.kind)
    out, off = [], 0
    for e in sp.entries:
        out.append(Proj(data[off * rb:(off + e.rows) * rb], e.rows, e.cols, e.kind, e.bias, e.rshift))
        off += e.rows
    return out


def gather(v, group=None):
    """All-gather of a 1-D float32 array in rank order."""
    t = torch.from_numpy(np.ascontiguousarray(v, dtype=f32))
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, t, group=group)
    return torch.cat(parts).numpy()


class OracleTP:
    def __init__(self, tpw, max_pos, group=None):
        cfg = self.cfg = tpw.cfg
        self.w, self.group = tpw, group
        host = lambda t: t.detach().cpu().numpy()
        self.emb = host(tpw.emb).astype(f32)
        self.out_norm = host(tpw.out_norm)
        self.freq = host(tpw.rope_freq)
        self.lm = _single(tpw.lm_head)
        self.layers = []
        for l, lw in enumerate(tpw.layers):
            sh = lw["shard"]
            d = {"attn_norm": host(lw["attn_norm"]), "ffn_norm": host(lw["ffn_norm"]), "in": _segments(lw["in"]),
                 "out": _single(lw["out"]), "gate": _single(lw["gate"]), "up": _single(lw["up"]),
                 "down": _single(lw["down"]), "shard": sh}
            if cfg.layer_type(l) == "d":
                for k in ("conv_w", "ssm_a", "dt_bias", "ssm_norm"):
                    d[k] = host(lw[k])
                d["win"] = np.zeros((cfg.dn_conv - 1, len(sh.channels)), f32)
                d["S"] = np.zeros((sh.nv, cfg.dn_hv, cfg.dn_hk), f32)
            else:
                d["q_norm"], d["k_norm"] = host(lw["q_norm"]), host(lw["k_norm"])
                d["kc"] = np.zeros((max_pos, sh.n_kv, cfg.head_dim), np.float16)
                d["vc"] = np.zeros((max_pos, sh.n_kv, cfg.head_dim), np.float16)
            self.layers.append(d)
        self.pos = 0

    def set_states(self, full_states):
        """DeltaNet states {layer: (nv, hv, hk) global array}: this rank's heads."""
        for l, s in full_states.items():
            self.layers[l]["S"][:] = s[self.layers[l]["shard"].heads]

    def forward(self, tok):
        cfg, eps, w = self.cfg, self.cfg.eps, self.w
        x = self.emb[tok].copy()
        for l, d in enumerate(self.layers):
            sh = d["shard"]
            hn = ref.rmsnorm(x, d["attn_norm"], eps)
            if cfg.layer_type(l) == "d":
                qkv, z, beta, alpha = (p(hn) for p in d["in"])
                og = ref.deltanet_step(qkv, z, beta, alpha, d["dt_bias"], d["ssm_a"], d["conv_w"], d["win"], d["S"],
                                       d["ssm_norm"], eps, sh.nk, cfg.dn_hk, sh.nv, cfg.dn_hv)
                y = d["out"](gather(og, self.group))
            else:
                qf, k, v = (p(hn) for p in d["in"])
                hd = cfg.head_dim
                if cfg.attn_gated:
                    qf = qf.reshape(sh.n_head, 2 * hd)
                    q, gate = qf[:, :hd].copy(), qf[:, hd:].copy()
                else:
                    q, gate = qf.reshape(sh.n_head, hd), None
                a = ref.attn_decode(q, k.reshape(sh.n_kv, hd), v.reshape(sh.n_kv, hd), d["kc"], d["vc"], self.pos,
                                    d["q_norm"], d["k_norm"], eps, self.freq, gate=gate)
                y = d["out"](gather(a.reshape(-1), self.group))
            x = gather((x[w.e0:w.e1] + y).astype(f32), self.group)
            hn = ref.rmsnorm(x, d["ffn_norm"], eps)
            act = gather((ref.silu(d["gate"](hn)) * d["up"](hn)).astype(f32), self.group)
            x = gather((x[w.e0:w.e1] + d["down"](act)).astype(f32), self.group)
        self.pos += 1
        logits = self.lm(ref.rmsnorm(x, self.out_norm, eps))
        i = ref.argmax_first(logits)
        best = torch.tensor([float(logits[i]), float(w.v0 + i)], dtype=torch.float64)
        parts = [torch.empty_like(best) for _ in range(dist.get_world_size(self.group))]
        dist.all_gather(parts, best, group=self.group)
        vals = [(float(p[0]), int(p[1])) for p in parts]
        top = max(v for v, _ in vals)
        return min(r for v, r in vals if v == top)

    def generate(self, prompt, n_new):
        tok = None
        for t in prompt:
            tok = self.forward(t)
        out = []
        for i in range(n_new):
            out.append(tok)
            if i + 1 < n_new:
                tok = self.forward(tok)
        return out
