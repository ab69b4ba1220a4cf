"""Decoder step of the reference engine restated on the CPU.  TEST INFRASTRUCTURE ONLY.

model/mirror.py:1002-1034 (`forward`, mathematical profile):
- the projections are the engine's float projection (quantise -> integer matvec -> scale) in
  the C oracle (oracle/trx_oracle.c), bit-exact with model/bitexact.py;
- attention is oracle/ref.py:attn_decode (mirror.py:945-996) with an fp16 KV cache;
- DeltaNet is oracle/ref.py:deltanet_step (mirror.py:892-943);
- RMSNorm, SiLU and argmax are oracle/ref.py.

Weights are host copies of a trixium_b200.decoder.SyntheticWeights (the same row-packet bytes
and B/R entries), so both sides decode the identical image.
"""

import numpy as np

from . import build as cor
from . import ref

f32 = np.float32


class Proj:
    def __init__(self, packed, rows, cols, kind, B, R):
        self.packed, self.rows, self.cols, self.kind, self.B, self.R = packed, rows, cols, kind, B, R

    def __call__(self, x):
        y, bad = cor.matvec_f(self.packed, self.rows, self.cols, self.kind, self.B, self.R,
                              np.ascontiguousarray(x, dtype=f32))
        assert bad == 0, "int48 accumulator or int32 result overflow"
        return y


def _segments(packed_group):
    """Proj per segment of a trixium_b200.decoder.Packed."""
    from trixium_b200 import layout as L
    data = packed_group.data.cpu().numpy()
    rb = L.row_bytes(packed_group.cols, packed_group.kind)
    out, off = [], 0
    for e in packed_group.entries:
        out.append(Proj(data[off * rb:(off + e.rows) * rb], e.rows, e.cols, e.kind, e.bias, e.rshift))
        off += e.rows
    return out


def _single(dt):
    return Proj(dt.data.cpu().numpy(), dt.rows, dt.cols, dt.kind, dt.bias, dt.rshift)


class OracleModel:
    def __init__(self, weights, max_pos):
        cfg = self.cfg = weights.cfg
        host = lambda t: t.detach().cpu().numpy()
        self.emb = host(weights.emb).astype(f32)
        self.out_norm = host(weights.out_norm)
        self.lm = _single(weights.lm_head)
        self.freq = host(weights.rope_freq)
        self.layers = []
        for l, lw in enumerate(weights.layers):
            d = {"attn_norm": host(lw["attn_norm"]), "ffn_norm": host(lw["ffn_norm"]), "in": _segments(lw["in"]),
                 "out": _single(lw["out"]), "gate": _single(lw["gate"]), "up": _single(lw["up"]),
                 "down": _single(lw["down"])}
            if cfg.layer_type(l) == "d":
                for k in ("conv_w", "ssm_a", "dt_bias", "ssm_norm"):
                    d[k] = host(lw[k])
                d["win"] = np.zeros((cfg.dn_conv - 1, cfg.dn_channels), f32)
                d["S"] = np.zeros((cfg.dn_nv, cfg.dn_hv, cfg.dn_hk), f32)
            else:
                d["q_norm"], d["k_norm"] = host(lw["q_norm"]), host(lw["k_norm"])
                d["kc"] = np.zeros((max_pos, cfg.n_kv, cfg.head_dim), np.float16)
                d["vc"] = np.zeros((max_pos, cfg.n_kv, cfg.head_dim), np.float16)
            self.layers.append(d)
        self.pos = 0

    def set_states(self, states):
        """DeltaNet states {layer: (nv, hv, hk) array} (copies of the device's)."""
        for l, s in states.items():
            self.layers[l]["S"][:] = s

    def forward(self, tok):
        """One step (mirror.py forward): returns the greedy next token."""
        cfg, eps = self.cfg, self.cfg.eps
        x = self.emb[tok].copy()
        for l, d in enumerate(self.layers):
            hn = ref.rmsnorm(x, d["attn_norm"], eps)
            if cfg.layer_type(l) == "d":
                qkv, z, beta, alpha = (p(hn) for p in d["in"])
                og = ref.deltanet_step(qkv, z, beta, alpha, d["dt_bias"], d["ssm_a"], d["conv_w"], d["win"], d["S"],
                                       d["ssm_norm"], eps, cfg.dn_nk, cfg.dn_hk, cfg.dn_nv, cfg.dn_hv)
                y = d["out"](og)
            else:
                qf, k, v = (p(hn) for p in d["in"])
                H, hd = cfg.n_head, cfg.head_dim
                if cfg.attn_gated:
                    qf = qf.reshape(H, 2 * hd)
                    q, gate = qf[:, :hd].copy(), qf[:, hd:].copy()
                else:
                    q, gate = qf.reshape(H, hd), None
                a = ref.attn_decode(q, k.reshape(cfg.n_kv, hd), v.reshape(cfg.n_kv, hd), d["kc"], d["vc"], self.pos,
                                    d["q_norm"], d["k_norm"], eps, self.freq, gate=gate)
                y = d["out"](a.reshape(-1))
            x = (x + y).astype(f32)
            hn = ref.rmsnorm(x, d["ffn_norm"], eps)
            act = (ref.silu(d["gate"](hn)) * d["up"](hn)).astype(f32)
            x = (x + d["down"](act)).astype(f32)
        self.pos += 1
        logits = self.lm(ref.rmsnorm(x, self.out_norm, eps))
        return ref.argmax_first(logits)

    def generate(self, prompt, n_new):
        """mirror.py:1036-1044."""
        tok = None
        for t in prompt:
            tok = self.forward(t)
        out = []
        for i in range(n_new):
            out.append(tok)
            if i + 1 < n_new:
                tok = self.forward(tok)
        return out
