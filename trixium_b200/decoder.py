"""Batch-1 greedy decoding of the TriXium model families on the B200.

The token step follows model/mirror.py:1002-1034 (`forward`):

    x = embed(token)
    per layer: hn = RMSNorm(x);  y = DeltaNet(hn) or Attention(hn);  x += y
               hn = RMSNorm(x);  x += down(silu(gate(hn)) * up(hn))
    token = argmax(lm_head(RMSNorm(x)))

Every operation is a kernel of libtrixium_b200.so:
- projections sharing an input run as one segmented launch with the RMSNorm fused in front;
- residual adds are fused into the projection that produces y;
- gate/up run as one SwiGLU launch;
- the greedy token is written on the device by the LM-head launch;
- the position advances on the device.

One step is captured as a CUDA graph and replayed per token, and the token feeds back through
device memory, so decoding makes no host round trip.

Weights are synthetic and random-init. Every matrix is group-128 ternary in the converter's row
packets, drawn from the config-0 distribution (P(w=0)=0.4, fp16 scales |N(0,1)|*0.02). DeltaNet's
conv taps, A and dt bias follow model/tinygen.py:107-113.
"""

from dataclasses import dataclass
import math

import numpy as np
import torch

from . import _lib, ops
from . import layout as L
from .image import pack_rows_torch, synthetic_codes_scales_torch


@dataclass(frozen=True)
class DecoderConfig:
    name: str
    n_layer: int
    hidden: int
    n_head: int
    n_kv: int
    head_dim: int
    ffn: int
    vocab: int
    kind: int = L.KIND_TERNARY5
    rope_theta: float = 1e6
    rope_dims: int = 0            # rotated dims per head (0: all)
    attn_gated: bool = False      # q projection also emits a per-head output gate (Qwen3.5)
    pattern: str = ""             # per layer 'd' (gated DeltaNet) or 'a' (attention); "" = all 'a'
    dn_nk: int = 0
    dn_hk: int = 0
    dn_nv: int = 0
    dn_hv: int = 0
    dn_conv: int = 4
    eps: float = 1e-6

    def layer_type(self, l):
        return self.pattern[l] if self.pattern else "a"

    @property
    def q_rows(self):
        return self.n_head * self.head_dim * (2 if self.attn_gated else 1)

    @property
    def kv_rows(self):
        return self.n_kv * self.head_dim

    @property
    def dn_channels(self):
        return 2 * self.dn_nk * self.dn_hk + self.dn_nv * self.dn_hv

    def weight_bytes_per_token(self):
        """Bytes of ternary weights + scales streamed per token (row packets, padding included)."""
        rb = lambda cols: L.row_bytes(cols, self.kind)
        E, total = self.hidden, 0
        for l in range(self.n_layer):
            if self.layer_type(l) == "d":
                total += (self.dn_channels + 2 * self.dn_nv + self.dn_nv * self.dn_hv) * rb(E)
                total += E * rb(self.dn_nv * self.dn_hv)
            else:
                total += (self.q_rows + 2 * self.kv_rows) * rb(E) + E * rb(self.n_head * self.head_dim)
            total += 2 * self.ffn * rb(E) + E * rb(self.ffn)
        return total + self.vocab * rb(E)


def _hybrid_pattern(n_layer):
    return "".join("a" if (l % 4) == 3 else "d" for l in range(n_layer))


CONFIGS = {
    # Qwen3-1.7B shape, trit5.
    "qwen3-1.7b": DecoderConfig("qwen3-1.7b", 28, 2048, 16, 8, 128, 6144, 151936, L.KIND_TERNARY5),
    # Qwen3-8B shape, 2-bit image.
    "qwen3-8b": DecoderConfig("qwen3-8b", 36, 4096, 32, 8, 128, 12288, 151936, L.KIND_TERNARY),
    # Qwen3.5-style hybrid 2B: 3 DeltaNet : 1 attention, trit5.
    "hybrid-2b": DecoderConfig("hybrid-2b", 24, 2048, 16, 4, 256, 6144, 151936, L.KIND_TERNARY5,
                               rope_theta=1e7, rope_dims=64, attn_gated=True, pattern=_hybrid_pattern(24),
                               dn_nk=16, dn_hk=128, dn_nv=16, dn_hv=128, dn_conv=4),
    # Qwen3.5-style hybrid 27B, 2-bit image.
    "hybrid-27b": DecoderConfig("hybrid-27b", 64, 5120, 24, 4, 256, 17408, 151936, L.KIND_TERNARY,
                                rope_theta=1e7, rope_dims=64, attn_gated=True, pattern=_hybrid_pattern(64),
                                dn_nk=16, dn_hk=128, dn_nv=48, dn_hv=128, dn_conv=4),
    # Small shapes for parity tests against the oracle model.
    "tiny": DecoderConfig("tiny", 2, 256, 4, 2, 64, 512, 1000, L.KIND_TERNARY5),
    # One kv head: tensor parallelism replicates it on every rank.
    "tiny-kv1": DecoderConfig("tiny-kv1", 2, 256, 4, 1, 64, 512, 1000, L.KIND_TERNARY),
    # Head dim 256 with one kv head and 6 query heads: over two ranks each holds the kv head and
    # 3 query heads, the shape config 4 has on 8 GPUs (the scratch-merge attention kernel).
    "tiny-hd256": DecoderConfig("tiny-hd256", 2, 256, 6, 1, 256, 512, 1000, L.KIND_TERNARY, rope_dims=64,
                                attn_gated=True),
    # An ffn wider than one tensor: the down projection is K-segmented (two segments, 8192 + 8320 columns).
    "tiny-kseg": DecoderConfig("tiny-kseg", 2, 256, 4, 2, 64, 16512, 1000, L.KIND_TERNARY),
    "tiny-hybrid": DecoderConfig("tiny-hybrid", 4, 256, 4, 2, 64, 512, 1000, L.KIND_TERNARY, rope_dims=32,
                                 attn_gated=True, pattern="dda" + "a", dn_nk=2, dn_hk=64, dn_nv=4, dn_hv=64,
                                 dn_conv=4),
}


# Weights --------------------------------------------------------------------------------------------

def _fp16_parts_torch(scales):
    b = scales.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    E = (b >> 10) & 31
    mant = b & 0x3FF
    m11 = torch.where(E == 0, mant, mant | 0x400)
    e16 = torch.where(E == 0, torch.full_like(E, -24), E - 25)
    return m11, e16


def _bias_rshift(scales_list, gs_max=128 * 127, target_top=12):
    """model/bitexact.py:77-97 (choose_scale_bias / choose_result_shift) over device scales."""
    B = target_top - max(int(_fp16_parts_torch(s)[1].max()) for s in scales_list)
    bound = 0.0
    for s in scales_list:
        m11, e16 = _fp16_parts_torch(s)
        per = torch.ceil(m11.double() * gs_max * torch.exp2((e16 + B).double()))
        bound = max(bound, float(per.sum(dim=-1).max()))
    R = 0
    while bound / float(1 << R) >= 2.0 ** 31:
        R += 1
    return B, R


class Packed:
    """Tensors sharing one input, their row packets back to back (one segmented launch)."""

    def __init__(self, gen, segments, cols, kind, device, chunk_rows=16384):
        self.names = [n for n, _ in segments]
        self.rows = [r for _, r in segments]
        self.cols, self.kind = cols, kind
        rb = L.row_bytes(cols, kind)
        self.data = torch.empty(sum(self.rows) * rb, dtype=torch.uint8, device=device)
        self.entries, off = [], 0
        for _, rows in segments:
            scales = []
            for r0 in range(0, rows, chunk_rows):
                n = min(chunk_rows, rows - r0)
                codes, sc = synthetic_codes_scales_torch(gen, n, cols, device)
                self.data[(off + r0) * rb:(off + r0 + n) * rb] = pack_rows_torch(sc, codes, kind)
                scales.append(sc)
            B, R = _bias_rshift(scales)
            self.entries.append(_lib.Entry(rows, cols, kind, B, R))
            off += rows

    def tensor(self, i):
        """Segment i as a DeviceTensor (a view of the shared allocation)."""
        rb = L.row_bytes(self.cols, self.kind)
        off = sum(self.rows[:i]) * rb
        e = self.entries[i]
        return ops.DeviceTensor.from_packed(self.data[off:off + self.rows[i] * rb], e.rows, e.cols, e.kind,
                                            e.bias, e.rshift)


KSEG_MAX = 16384  # the widest K one engine op takes (model/layout.py:94)


def ksegmented(gen, rows, cols, kind, device, kseg_max=KSEG_MAX):
    """A tensor wider than kseg_max as the converter stores it (model/bons.py:83-113 split_wide):
    K-segments over equal column ranges (a multiple of the group each), the whole tensor's B and R in
    every segment, each segment its own row packets.  Returns the segments' DeviceTensors in order."""
    nseg = -(-cols // kseg_max)
    G = cols // L.GROUP
    bounds = [(G * k // nseg) * L.GROUP for k in range(nseg + 1)]
    codes, scales = synthetic_codes_scales_torch(gen, rows, cols, device)
    B, R = _bias_rshift([scales])
    segs = []
    for k in range(nseg):
        c0, c1 = bounds[k], bounds[k + 1]
        packed = pack_rows_torch(scales[:, c0 // L.GROUP:c1 // L.GROUP].contiguous(), codes[:, c0:c1].contiguous(), kind)
        segs.append(ops.DeviceTensor.from_packed(packed, rows, c1 - c0, kind, B, R))
    return segs


class SyntheticWeights:
    """Random-init weights of a DecoderConfig, resident on the device.  A matrix wider than one
    engine op (K > 16384: the hybrid-27b down projection) is stored K-segmented as the converter
    stores it, a list of its segments."""

    def __init__(self, cfg: DecoderConfig, seed=0, device="cuda"):
        self.cfg = cfg
        dev = torch.device(device)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        rng = np.random.default_rng(seed)
        E, kind = cfg.hidden, cfg.kind
        norm = lambda n: torch.from_numpy((1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)).to(dev)
        self.emb = (torch.randn(cfg.vocab, E, generator=gen, device=dev)).to(torch.float16)
        self.layers = []
        for l in range(cfg.n_layer):
            w = {"attn_norm": norm(E), "ffn_norm": norm(E)}
            if cfg.layer_type(l) == "d":
                nv, hv, C = cfg.dn_nv, cfg.dn_hv, cfg.dn_channels
                w["in"] = Packed(gen, [("qkv", C), ("z", nv * hv), ("beta", nv), ("alpha", nv)], E, kind, dev)
                w["out"] = Packed(gen, [("ssm_out", E)], nv * hv, kind, dev).tensor(0)
                f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)
                w["conv_w"] = f32(rng.uniform(-0.5, 0.5, (C, cfg.dn_conv)))
                w["ssm_a"] = f32(-np.exp(rng.uniform(-1.5, 0.5, nv)))
                w["dt_bias"] = f32(rng.uniform(-2.0, 0.5, nv))
                w["ssm_norm"] = norm(hv)
            else:
                w["in"] = Packed(gen, [("q", cfg.q_rows), ("k", cfg.kv_rows), ("v", cfg.kv_rows)], E, kind, dev)
                w["out"] = Packed(gen, [("o", E)], cfg.n_head * cfg.head_dim, kind, dev).tensor(0)
                w["q_norm"] = norm(cfg.head_dim)
                w["k_norm"] = norm(cfg.head_dim)
            ffn = Packed(gen, [("gate", cfg.ffn), ("up", cfg.ffn)], E, kind, dev)
            w["gate"], w["up"] = ffn.tensor(0), ffn.tensor(1)
            w["ffn_packed"] = ffn
            w["down"] = (ksegmented(gen, E, cfg.ffn, kind, dev) if cfg.ffn > KSEG_MAX
                         else Packed(gen, [("down", E)], cfg.ffn, kind, dev).tensor(0))
            self.layers.append(w)
        self.out_norm = norm(E)
        self.lm_head = Packed(gen, [("lm_head", cfg.vocab)], E, kind, dev).tensor(0)
        rope_n = cfg.rope_dims or cfg.head_dim
        self.rope_freq = torch.from_numpy(np.array(
            [np.float32(np.float32(cfg.rope_theta) ** np.float32(-2.0 * i / rope_n)) for i in range(rope_n // 2)],
            dtype=np.float32)).to(dev)


# The decoder ------------------------------------------------------------------------------------------

class Decoder:
    """Greedy batch-1 decoding over SyntheticWeights (or any weights of the same layout)."""

    def __init__(self, weights: SyntheticWeights, ctx=None, max_pos=4096, kv_dtype=torch.float16):
        cfg = self.cfg = weights.cfg
        self.w = weights
        self.ctx = ctx or ops.default_context()
        dev = weights.emb.device
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)
        E = cfg.hidden
        self.max_pos = max_pos
        self.x = f32(E)
        self.q, self.k, self.v = f32(cfg.q_rows), f32(cfg.kv_rows), f32(cfg.kv_rows)
        self.attn = f32(cfg.n_head * cfg.head_dim)
        self.act = f32(cfg.ffn)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.attn_shape = ops.attn_shape(cfg.n_head, cfg.n_kv, cfg.head_dim, max_pos,
                                         rope_dims=cfg.rope_dims or cfg.head_dim, gated=cfg.attn_gated, eps=cfg.eps)
        self.kc, self.vc, self.ring, self.state = {}, {}, {}, {}
        for l in range(cfg.n_layer):
            if cfg.layer_type(l) == "d":
                self.ring[l] = f32(cfg.dn_conv * cfg.dn_channels).view(cfg.dn_conv, cfg.dn_channels)
                self.state[l] = f32(cfg.dn_nv * cfg.dn_hv * cfg.dn_hk).view(cfg.dn_nv, cfg.dn_hv, cfg.dn_hk)
            else:
                self.kc[l] = torch.zeros(max_pos, cfg.n_kv, cfg.head_dim, dtype=kv_dtype, device=dev)
                self.vc[l] = torch.zeros_like(self.kc[l])
        if any(cfg.layer_type(l) == "d" for l in range(cfg.n_layer)):
            self.dn_shape = ops.deltanet_shape(cfg.dn_nk, cfg.dn_hk, cfg.dn_nv, cfg.dn_hv, cfg.dn_conv, cfg.eps)
            self.qkv, self.z = f32(cfg.dn_channels), f32(cfg.dn_nv * cfg.dn_hv)
            self.beta, self.alpha = f32(cfg.dn_nv), f32(cfg.dn_nv)
            self.og = f32(cfg.dn_nv * cfg.dn_hv)
        self.graph = None

    def _mutable(self):
        return [self.tok, self.pos] + list(self.kc.values()) + list(self.vc.values()) + list(self.ring.values()) + \
            list(self.state.values())

    def reset(self):
        """Empty caches and states, position 0."""
        self.pos.zero_()
        for t in list(self.kc.values()) + list(self.vc.values()) + list(self.ring.values()) + list(self.state.values()):
            t.zero_()

    def set_states(self, seed=0):
        """Random DeltaNet states ~N(0,1)/sqrt(hk) (BASELINE's recurrent init)."""
        g = torch.Generator(device=self.tok.device)
        g.manual_seed(seed)
        for t in self.state.values():
            t.copy_(torch.randn(t.shape, generator=g, device=t.device) / math.sqrt(self.cfg.dn_hk))

    def fill_context(self, n, seed=0):
        """Synthetic context of n positions: random fp16 K/V rows in every attention cache (of the
        scale the step's normalised keys have) and the position set to n."""
        g = torch.Generator(device=self.tok.device)
        g.manual_seed(seed)
        for l in self.kc:
            self.kc[l][:n] = torch.randn(self.kc[l][:n].shape, generator=g, device=self.tok.device).to(self.kc[l].dtype)
            self.vc[l][:n] = torch.randn(self.vc[l][:n].shape, generator=g, device=self.tok.device).to(self.vc[l].dtype)
        self.pos.fill_(n)

    def enqueue_step(self):
        """One token's kernels on the current stream: reads self.tok and self.pos, writes the next
        token into self.tok and advances self.pos."""
        cfg, w, ctx = self.cfg, self.w, self.ctx
        ops.embed_lookup(ctx, w.emb, self.tok, self.x)
        for l, lw in enumerate(w.layers):
            p = lw["in"]
            if cfg.layer_type(l) == "d":
                ops.matvec_f_multi(ctx, p.entries, p.data, self.x, [self.qkv, self.z, self.beta, self.alpha],
                                   norm_w=lw["attn_norm"], eps=cfg.eps)
                ops.deltanet_step(ctx, self.dn_shape, self.qkv, self.z, self.beta, self.alpha, lw["dt_bias"],
                                  lw["ssm_a"], lw["conv_w"], lw["ssm_norm"], self.ring[l], self.state[l], self.pos,
                                  self.og)
                ops.matvec_f(ctx, lw["out"], self.og, y=self.x, resid=self.x)
            else:
                ops.matvec_f_multi(ctx, p.entries, p.data, self.x, [self.q, self.k, self.v], norm_w=lw["attn_norm"],
                                   eps=cfg.eps)
                ops.attn_decode(ctx, self.attn_shape, self.q, self.k, self.v, lw["q_norm"], lw["k_norm"], w.rope_freq,
                                self.kc[l], self.vc[l], self.pos, self.attn)
                ops.matvec_f(ctx, lw["out"], self.attn, y=self.x, resid=self.x)
            ops.matvec_swiglu(ctx, lw["gate"], lw["up"], self.x, act=self.act, norm_w=lw["ffn_norm"], eps=cfg.eps)
            if isinstance(lw["down"], list):  # K-segmented
                ops.matvec_f_kseg(ctx, lw["down"], self.act, y=self.x, resid=self.x)
            else:
                ops.matvec_f(ctx, lw["down"], self.act, y=self.x, resid=self.x)
        ops.lmhead_argmax(ctx, w.lm_head, self.x, token=self.tok, norm_w=w.out_norm, eps=cfg.eps)
        ops.advance_position(ctx, self.pos)

    def launches_per_step(self):
        # embedding; per layer 5 (input projections, attention or DeltaNet, output projection,
        # gate/up, down), a K-segmented down projection one launch per segment, plus the quantiser
        # and the combine unless it has two ternary segments (trx_matvec_f_kseg); LM head and
        # position advance.
        def kseg_launches(segs):
            two = len(segs) == 2 and all(t.kind != L.KIND_Q8 for t in segs)
            return len(segs) + (0 if two else 2)

        n = 1 + 2
        for lw in self.w.layers:
            n += 4 + (kseg_launches(lw["down"]) if isinstance(lw["down"], list) else 1)
        return n

    def capture(self):
        """Capture one step as a CUDA graph (the kernels read the position on the device)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        live = self._mutable()
        saved = [t.clone() for t in live]
        with torch.cuda.stream(s):
            self.enqueue_step()          # warm-up outside the capture, then every buffer restored
            torch.cuda.synchronize()
        for t, c in zip(live, saved):
            t.copy_(c)
        del saved
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self.enqueue_step()
        torch.cuda.synchronize()
        return self.graph

    def step(self, token=None):
        """One token: feed `token` (teacher forcing) or the previous step's greedy token."""
        if token is not None:
            self.tok.fill_(int(token))
        if self.graph is not None:
            self.graph.replay()
        else:
            self.enqueue_step()

    def generate(self, prompt, n_new):
        """Greedy decode: the prompt, then n_new tokens (mirror.py:1036-1042).  Returns the new ids."""
        for t in prompt:
            self.step(t)
        out = torch.empty(n_new, dtype=torch.int32, device=self.tok.device)
        for i in range(n_new):
            out[i:i + 1].copy_(self.tok)
            if i + 1 < n_new:  # no unused step after the final output (mirror.py:1042)
                self.step()
        self.ctx.raise_on_error()
        return out.cpu().tolist()


class BatchDecoder:
    """Greedy decoding of nseq <= 32 independent sequences in lockstep (BASELINE config 2 at batch
    16): the tensors sharing an input run as one tensor-core launch over the sequences' rows
    (trx_matvec_f_rows_multi: q/k/v or qkv/z/beta/alpha, gate/up; the RMSNorm in front, each row
    quantised with its own exponent as the batch-1 projection quantises its vector), the output and
    down projections add the residual, SwiGLU, the final norm, argmax and position advance are
    row-wise kernels, and attention and the DeltaNet step run over a sequence grid dimension with
    per-sequence caches, states and positions.  The arithmetic of every sequence is the batch-1
    decoder's (mirror.py:1002-1034).  A K-segmented down projection (hybrid-27b) of two ternary
    segments takes trx_matvec_f_rows_kseg: one exponent per sequence over the whole act."""

    def __init__(self, weights: SyntheticWeights, nseq, ctx=None, max_pos=4096, kv_dtype=torch.float16):
        cfg = self.cfg = weights.cfg
        if not 1 <= nseq <= 32:
            raise ValueError("BatchDecoder: 1 <= nseq <= 32")
        for lw in weights.layers:
            d = lw["down"]
            if isinstance(d, list) and (len(d) != 2 or any(t.kind == L.KIND_Q8 for t in d)):
                raise ValueError("BatchDecoder: a K-segmented tensor needs two ternary segments")
        self.w, self.nseq = weights, nseq
        self.ctx = ctx or ops.default_context()
        dev = weights.emb.device
        f32 = lambda *shape: torch.zeros(*shape, dtype=torch.float32, device=dev)
        E, B = cfg.hidden, nseq
        self.max_pos = max_pos
        self.x, self.h = f32(B, E), f32(B, E)
        self.q, self.k, self.v = f32(B, cfg.q_rows), f32(B, cfg.kv_rows), f32(B, cfg.kv_rows)
        self.attn = f32(B, cfg.n_head * cfg.head_dim)
        self.g, self.u, self.act = f32(B, cfg.ffn), f32(B, cfg.ffn), f32(B, cfg.ffn)
        self.logits = f32(B, cfg.vocab)
        self.tok = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.attn_shape = ops.attn_shape(cfg.n_head, cfg.n_kv, cfg.head_dim, max_pos,
                                         rope_dims=cfg.rope_dims or cfg.head_dim, gated=cfg.attn_gated, eps=cfg.eps)
        self.kc, self.vc, self.ring, self.state = {}, {}, {}, {}
        for l in range(cfg.n_layer):
            if cfg.layer_type(l) == "d":
                self.ring[l] = f32(B, cfg.dn_conv, cfg.dn_channels)
                self.state[l] = f32(B, cfg.dn_nv, cfg.dn_hv, cfg.dn_hk)
            else:
                self.kc[l] = torch.zeros(B, max_pos, cfg.n_kv, cfg.head_dim, dtype=kv_dtype, device=dev)
                self.vc[l] = torch.zeros_like(self.kc[l])
        if self.ring:
            self.dn_shape = ops.deltanet_shape(cfg.dn_nk, cfg.dn_hk, cfg.dn_nv, cfg.dn_hv, cfg.dn_conv, cfg.eps)
            self.qkv, self.z = f32(B, cfg.dn_channels), f32(B, cfg.dn_nv * cfg.dn_hv)
            self.beta, self.alpha = f32(B, cfg.dn_nv), f32(B, cfg.dn_nv)
            self.og = f32(B, cfg.dn_nv * cfg.dn_hv)
        self.graph = None

    def _mutable(self):
        return [self.tok, self.pos] + list(self.kc.values()) + list(self.vc.values()) + list(self.ring.values()) + \
            list(self.state.values())

    def set_states(self, states):
        """Every sequence's DeltaNet states: states[l] of shape (nv, hv, hk) (the batch-1 decoder's)."""
        for l, t in self.state.items():
            t.copy_(states[l].unsqueeze(0).expand_as(t))

    def fill_context(self, n, seed=0):
        """Synthetic context of n positions in every sequence's attention caches (random fp16 K/V
        rows) and every position set to n."""
        g = torch.Generator(device=self.tok.device)
        g.manual_seed(seed)
        for l in self.kc:
            self.kc[l][:, :n] = torch.randn(self.kc[l][:, :n].shape, generator=g, device=self.tok.device).to(self.kc[l].dtype)
            self.vc[l][:, :n] = torch.randn(self.vc[l][:, :n].shape, generator=g, device=self.tok.device).to(self.vc[l].dtype)
        self.pos.fill_(n)

    def enqueue_step(self):
        """One token of every sequence on the current stream: reads self.tok and self.pos, writes the
        next tokens into self.tok and advances self.pos."""
        cfg, w, ctx = self.cfg, self.w, self.ctx
        ops.embed_lookup_rows(ctx, w.emb, self.tok, self.x)
        for l, lw in enumerate(w.layers):
            p = lw["in"]
            if cfg.layer_type(l) == "d":
                ops.matvec_f_rows_multi(ctx, p.entries, p.data, self.x, [self.qkv, self.z, self.beta, self.alpha],
                                        norm_w=lw["attn_norm"], eps=cfg.eps)
                ops.deltanet_step_rows(ctx, self.dn_shape, self.qkv, self.z, self.beta, self.alpha, lw["dt_bias"],
                                       lw["ssm_a"], lw["conv_w"], lw["ssm_norm"], self.ring[l], self.state[l], self.pos,
                                       self.og)
                ops.matvec_f_rows(ctx, lw["out"], self.og, out=self.x, resid=self.x)
            else:
                ops.matvec_f_rows_multi(ctx, p.entries, p.data, self.x, [self.q, self.k, self.v],
                                        norm_w=lw["attn_norm"], eps=cfg.eps)
                ops.attn_decode_rows(ctx, self.attn_shape, self.q, self.k, self.v, lw["q_norm"], lw["k_norm"],
                                     w.rope_freq, self.kc[l], self.vc[l], self.pos, self.attn)
                ops.matvec_f_rows(ctx, lw["out"], self.attn, out=self.x, resid=self.x)
            ffn = lw["ffn_packed"]
            ops.matvec_f_rows_multi(ctx, ffn.entries, ffn.data, self.x, [self.g, self.u], norm_w=lw["ffn_norm"],
                                    eps=cfg.eps)
            ops.silu_mul(ctx, self.g, self.u, self.act)
            if isinstance(lw["down"], list):
                ops.matvec_f_rows_kseg(ctx, lw["down"], self.act, out=self.x, resid=self.x)
            else:
                ops.matvec_f_rows(ctx, lw["down"], self.act, out=self.x, resid=self.x)
        ops.rmsnorm_rows(ctx, self.x, w.out_norm, cfg.eps, y=self.h)
        ops.matvec_f_rows(ctx, w.lm_head, self.h, out=self.logits)
        ops.argmax_rows(ctx, self.logits, self.tok)
        ops.advance_positions(ctx, self.pos)

    def capture(self):
        """Capture one step as a CUDA graph (positions and tokens live on the device)."""
        return Decoder.capture(self)

    def step(self, tokens=None):
        if tokens is not None:
            self.tok.copy_(torch.as_tensor(tokens, dtype=torch.int32))
        if self.graph is not None:
            self.graph.replay()
        else:
            self.enqueue_step()

    def generate(self, prompts, n_new):
        """Greedy decode of every sequence: prompts [nseq][P] (equal lengths), then n_new tokens each.
        Returns [nseq][n_new] ids."""
        P = len(prompts[0])
        for t in range(P):
            self.step([p[t] for p in prompts])
        out = torch.empty(n_new, self.nseq, dtype=torch.int32, device=self.tok.device)
        for i in range(n_new):
            out[i].copy_(self.tok)
            if i + 1 < n_new:
                self.step()
        self.ctx.raise_on_error()
        return out.t().cpu().tolist()


def main(argv=None):
    """Decode timing on synthetic weights: python -m trixium_b200.decoder --config qwen3-8b
    --context 1024 --tokens 64 [--eager].  Prints one JSON line (ms and tok/s per token)."""
    import argparse
    import json
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--config", default="qwen3-8b", choices=sorted(CONFIGS))
    ap.add_argument("--context", type=int, default=1024)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--eager", action="store_true", help="launch the kernels directly (no CUDA graph)")
    a = ap.parse_args(argv)
    cfg = CONFIGS[a.config]
    dec = Decoder(SyntheticWeights(cfg, seed=0), max_pos=a.context + a.tokens + a.warmup + 8)
    dec.set_states(1)
    dec.fill_context(a.context)
    dec.tok.fill_(7)
    if not a.eager:
        dec.capture()
    for _ in range(a.warmup):
        dec.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.tokens):
        dec.step()
    e1.record()
    torch.cuda.synchronize()
    dec.ctx.raise_on_error()
    ms = e0.elapsed_time(e1) / a.tokens
    print(json.dumps({"config": a.config, "context": a.context, "tokens": a.tokens, "graph": not a.eager,
                      "ms_per_token": round(ms, 4), "tok_s": round(1000.0 / ms, 1),
                      "launches_per_token": dec.launches_per_step()}))


if __name__ == "__main__":
    main()


# Decoding from a BONS image ---------------------------------------------------------------------------

class ImageWeights:
    """The weights of a BONS image (trixium_b200.bons.BONSImage) on the device, as the reference's
    firmware mirror reads them (model/mirror.py:594-800): every matvec tensor with its entry's B and
    R (K-segmented tensors as their segments, FLAG_KSEG), the rotation block tensors of every input
    width (ROLE_HADAMARD, stacked per width), the F32 norm weights, conv taps, A and dt bias, and the
    int16 embedding table.  `cfg` is the DecoderConfig the header describes."""

    def __init__(self, img, device="cuda"):
        from . import bons as Bn
        dev = torch.device(device)
        h = self.header = img.header
        E, H, Hkv, hd = h["n_embd"], h["n_head"], h["n_kv_head"], h["head_dim"]
        dn = [t == "deltanet" for t in h["layer_types"]]
        self.rot_block = h["hadamard_block"]
        self.cfg = DecoderConfig(
            "image", h["n_layer"], E, H, Hkv, hd, h["ffn_dim"], h["vocab"], L.KIND_TERNARY,
            rope_theta=float(np.float32(h["rope_theta"])), rope_dims=h["rope_dims"], attn_gated=bool(h["attn_gated"]),
            pattern="".join("d" if d else "a" for d in dn), dn_nk=h["dn_num_k_heads"], dn_hk=h["dn_k_head_dim"],
            dn_nv=h["dn_num_v_heads"], dn_hv=h["dn_v_head_dim"], dn_conv=h["dn_conv_kernel"] or 4,
            eps=float(np.float32(h["rms_eps"])))
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)

        def rows(role, l):
            return f32(img.plain_rows(img.entries_of(role, l, L.KIND_F32)[0]).reshape(-1))

        def mv(role, l=0):
            return [img.device_tensor(e, device=dev) for e in img.matvec_entries(role, l)]

        emb = img.embedding_bfp16()
        if emb is None:
            raise ValueError("the image has no int16 embedding table (ROLE_TOK_EMB16)")
        self.emb = torch.from_numpy(np.ascontiguousarray(emb[0])).to(dev)
        self.emb_exp = torch.from_numpy(np.ascontiguousarray(emb[1])).to(dev)
        # Rotation: per input width, its blocks' tensors back to back (one batched launch).
        self.rot = {}
        for wi, width in enumerate(h["hadamard_widths"] if self.rot_block else ()):
            blocks = [img.find(role=Bn.ROLE_HADAMARD, layer=Bn.hadamard_layer(wi, b))
                      for b in range(width // self.rot_block)]
            if len({(e["bias"], e["rshift"], e["kind"]) for e in blocks}) != 1:
                raise ValueError(f"rotation blocks of width {width} differ in B/R or kind")
            e0 = blocks[0]
            packed = np.concatenate([np.asarray(img.row_packets(e)) for e in blocks])
            self.rot[width] = ops.DeviceTensor.from_packed(packed, width, e0["cols"], e0["kind"], e0["bias"],
                                                           e0["rshift"], device=dev)
        self.layers = []
        for l in range(h["n_layer"]):
            w = {"attn_norm": rows(Bn.ROLE_ATTN_NORM, l), "ffn_norm": rows(Bn.ROLE_FFN_NORM, l)}
            if dn[l]:
                w.update(qkv=mv(Bn.ROLE_ATTN_QKV, l), z=mv(Bn.ROLE_ATTN_ZGATE, l), beta=mv(Bn.ROLE_SSM_BETA, l),
                         alpha=mv(Bn.ROLE_SSM_ALPHA, l), out=mv(Bn.ROLE_SSM_OUT, l),
                         conv_w=rows(Bn.ROLE_SSM_CONV, l), ssm_a=rows(Bn.ROLE_SSM_A, l),
                         dt_bias=rows(Bn.ROLE_SSM_DT, l), ssm_norm=rows(Bn.ROLE_SSM_NORM, l))
            else:
                w.update(q=mv(Bn.ROLE_ATTN_Q, l), k=mv(Bn.ROLE_ATTN_K, l), v=mv(Bn.ROLE_ATTN_V, l),
                         out=mv(Bn.ROLE_ATTN_OUT, l), q_norm=rows(Bn.ROLE_ATTN_Q_NORM, l),
                         k_norm=rows(Bn.ROLE_ATTN_K_NORM, l))
            w.update(gate=mv(Bn.ROLE_FFN_GATE, l), up=mv(Bn.ROLE_FFN_UP, l), down=mv(Bn.ROLE_FFN_DOWN, l))
            self.layers.append(w)
        self.out_norm = rows(Bn.ROLE_OUT_NORM, 0)
        head = img.entries_of(Bn.ROLE_LM_HEAD, 0) or img.entries_of(Bn.ROLE_TOK_EMB, 0)
        head = [e for e in head if e["kind"] in L.TERNARY_KINDS]
        if len(head) != 1:
            raise ValueError("the LM head must be one ternary tensor")
        lm = img.device_tensor(head[0], device=dev)
        V = h["vocab"]  # rows past the vocabulary are channel padding and never win (model/mirror.py:1030)
        self.lm_head = ops.DeviceTensor.from_packed(lm.data[:V * L.row_bytes(lm.cols, lm.kind)], V, lm.cols, lm.kind,
                                                    lm.bias, lm.rshift)
        rope_n = self.cfg.rope_dims or hd
        self.rope_freq = f32([np.float32(np.float32(h["rope_theta"]) ** np.float32(-2.0 * i / rope_n))
                              for i in range(rope_n // 2)])


class ImageDecoder(Decoder):
    """Greedy decoding of a BONS image in the reference mirror's engine arithmetic
    (model/mirror.py:594-1044, hybrid27_generate with exact=False, mathematical profile):
    per token, the int16 embedding row; per layer RMSNorm, the rotation of every projection's input
    (blockwise quantised projections, model/mirror.py:680-690), the projections (K-segmented ones
    summed after each segment's >> R), DeltaNet or gated attention, the residual adds, SwiGLU; then
    the LM head's greedy token.  `trace(layer, tag, tensor)`, eager steps only, receives the values the
    mirror's trace hook names (emb, attn_norm, attn_out/dn_out, attn_res, ffn_norm, ffn_act, ffn_res,
    out_norm).  kv_dtype float32 keeps the mirror's fp32 KV cache (trx_attn_decode_f32cache)."""

    def __init__(self, weights: ImageWeights, ctx=None, max_pos=512, kv_dtype=torch.float16):
        super().__init__(weights, ctx=ctx, max_pos=max_pos, kv_dtype=kv_dtype)
        cfg, dev = self.cfg, self.x.device
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)
        self.hn = f32(cfg.hidden)
        self.rin = f32(max(cfg.hidden, cfg.ffn, cfg.n_head * cfg.head_dim, cfg.dn_nv * cfg.dn_hv))
        self.logits = f32(cfg.vocab)
        self.trace = None

    def _rotate(self, x, width):
        if not self.w.rot_block:
            return x
        out = self.rin[:width]
        return ops.hadamard_rotate(self.ctx, self.w.rot[width], x, out=out)

    def _proj(self, segs, x, y, resid=None):
        if len(segs) > 1:
            return ops.matvec_f_kseg(self.ctx, segs, x, y=y, resid=resid)
        t = segs[0]
        if t.kind == L.KIND_Q8:
            if resid is not None:
                raise ValueError("a Q8 projection takes no residual")
            return ops.matvec_q8_f(self.ctx, t, x, out=y)
        return ops.matvec_f(self.ctx, t, x, y=y, resid=resid)

    def _tr(self, l, tag, t):
        if self.trace is not None:
            self.trace(l, tag, t.clone())

    def enqueue_step(self):
        cfg, w, ctx = self.cfg, self.w, self.ctx
        E = cfg.hidden
        ops.embed_lookup_bfp16(ctx, w.emb, w.emb_exp, self.tok, self.x)
        self._tr(-1, "emb", self.x)
        for l, lw in enumerate(w.layers):
            ops.rmsnorm(ctx, self.x, lw["attn_norm"], cfg.eps, y=self.hn)
            self._tr(l, "attn_norm", self.hn)
            r = self._rotate(self.hn, E)
            if cfg.layer_type(l) == "d":
                self._proj(lw["qkv"], r, self.qkv)
                self._proj(lw["z"], r, self.z)
                self._proj(lw["beta"], self.hn, self.beta)   # not rotated (model/mirror.py:895-896)
                self._proj(lw["alpha"], self.hn, self.alpha)
                ops.deltanet_step(ctx, self.dn_shape, self.qkv, self.z, self.beta, self.alpha, lw["dt_bias"],
                                  lw["ssm_a"], lw["conv_w"], lw["ssm_norm"], self.ring[l], self.state[l], self.pos,
                                  self.og)
                self._tr(l, "dn_og", self.og)
                self._proj(lw["out"], self._rotate(self.og, cfg.dn_nv * cfg.dn_hv), self.x, resid=self.x)
            else:
                self._proj(lw["q"], r, self.q)
                self._proj(lw["k"], r, self.k)
                self._proj(lw["v"], r, self.v)
                ops.attn_decode(ctx, self.attn_shape, self.q, self.k, self.v, lw["q_norm"], lw["k_norm"], w.rope_freq,
                                self.kc[l], self.vc[l], self.pos, self.attn)
                self._tr(l, "attn", self.attn)
                self._proj(lw["out"], self._rotate(self.attn, cfg.n_head * cfg.head_dim), self.x, resid=self.x)
            self._tr(l, "attn_res", self.x)
            ops.rmsnorm(ctx, self.x, lw["ffn_norm"], cfg.eps, y=self.hn)
            self._tr(l, "ffn_norm", self.hn)
            r = self._rotate(self.hn, E)
            if len(lw["gate"]) == 1 and len(lw["up"]) == 1:
                ops.matvec_swiglu(ctx, lw["gate"][0], lw["up"][0], r, act=self.act)
            else:
                raise ValueError("K-segmented gate/up projections (wider than one engine op) are not expected: "
                                 "their input is the hidden size")
            self._tr(l, "ffn_act", self.act)
            self._proj(lw["down"], self._rotate(self.act, cfg.ffn), self.x, resid=self.x)
            self._tr(l, "ffn_res", self.x)
        ops.rmsnorm(ctx, self.x, w.out_norm, cfg.eps, y=self.hn)
        self._tr(-1, "out_norm", self.hn)
        ops.lmhead_argmax(ctx, w.lm_head, self._rotate(self.hn, E), token=self.tok, logits=self.logits)
        ops.advance_position(ctx, self.pos)

    def launches_per_step(self):
        return None
