"""Tensor-parallel batch-1 decoding over N GPUs of one node (one process per GPU).

Every weight matrix is sharded by output rows (the reference's channel sharding,
model/layout.py:219-223). After each projection the ranks all-gather the output vector, so
every rank computes whole rows from the complete, identically quantised input, and the results
are bit-identical to one GPU. Splitting K instead would quantise each slice with its own exponent.

Per layer:
- **Attention:** rank r owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads: the rows of
  q/k/v, the KV cache and the attention of those heads are local. The head outputs are
  all-gathered in head order, then o-proj rows, residual and all-gather of x.
- **DeltaNet:** rank r owns key heads [r*nk/N, (r+1)*nk/N) and the value heads h with h % nk among
  them, renumbered locally so the kernel's tiled head map holds. Their grouped outputs
  (mirror.py:941-942) form one contiguous block of the layer output, all-gathered in rank order.
- **FFN:** gate/up rows, SwiGLU, all-gather of the activation, down rows, residual, all-gather x.
- **LM head:** vocabulary rows. Each rank's argmax key carries the global row; the keys are
  all-gathered and the largest one is the token (ties to the smallest row).

The plan functions below are pure index arithmetic, shared by the GPU engine (`TPDecoder`) and
the CPU tests that run the oracle sharded over gloo ranks.
"""

import numpy as np


def span(total, rank, world):
    """Rows [a, b) of `rank` in an even split of `total` (which `world` must divide)."""
    if total % world:
        raise ValueError(f"{total} rows do not split evenly over {world} ranks")
    n = total // world
    return rank * n, (rank + 1) * n


class AttnShard:
    """Rows of one rank's attention-layer shard (query rows per head: hd, or 2*hd when gated).

    With at least as many kv heads as ranks, rank r owns kv heads [kv0, kv1) and all their query
    heads.  With fewer (world a multiple of the kv heads, e.g. 4 kv heads on 8 GPUs), each kv head is
    replicated on g = world / n_kv ranks: the g ranks each compute that head's k/v rows and keep
    their own copy of its cache, and split its query heads evenly.  Either way rank r's query heads
    are [head0, head0 + n_head) with head0 = r * n_head, so the head outputs all-gather in rank
    order."""

    def __init__(self, cfg, rank, world):
        H, Hkv, hd = cfg.n_head, cfg.n_kv, cfg.head_dim
        rep = H // Hkv
        qh = hd * (2 if cfg.attn_gated else 1)
        if Hkv % world == 0:
            self.kv0, self.kv1 = span(Hkv, rank, world)
            self.n_kv = self.kv1 - self.kv0
            self.n_head = self.n_kv * rep
            self.head0 = self.kv0 * rep
            self.replicas = 1
        elif world % Hkv == 0 and rep % (world // Hkv) == 0:
            g = world // Hkv
            self.kv0 = rank // g
            self.kv1 = self.kv0 + 1
            self.n_kv = 1
            self.n_head = rep // g
            self.head0 = self.kv0 * rep + (rank % g) * self.n_head
            self.replicas = g
        else:
            raise ValueError(f"{Hkv} kv heads ({H} query heads) do not split over {world} ranks")
        self.q_rows = np.arange(self.head0 * qh, (self.head0 + self.n_head) * qh)
        self.k_rows = np.arange(self.kv0 * hd, self.kv1 * hd)
        self.v_rows = self.k_rows.copy()


class DeltaNetShard:
    """Channels and value heads of one rank's DeltaNet-layer shard.

    Local value head h' = (kh - k0) + m * nk' holds global head h = kh + m * nk (kh a local key
    head, m < nv/nk), so the kernel's map h' % nk' = kh - k0 is the global map h % nk = kh."""

    def __init__(self, cfg, rank, world):
        nk, hk, nv, hv = cfg.dn_nk, cfg.dn_hk, cfg.dn_nv, cfg.dn_hv
        if nk % world:
            raise ValueError(f"{nk} key heads do not split over {world} ranks")
        rep = nv // nk
        self.k0, self.k1 = span(nk, rank, world)
        self.nk = self.k1 - self.k0
        self.nv = self.nk * rep
        nq = nk * hk
        # Global value head of each local value head h' = (kh - k0) + m * nk'.
        self.heads = np.array([self.k0 + (hl % self.nk) + (hl // self.nk) * nk for hl in range(self.nv)])
        q = np.arange(self.k0 * hk, self.k1 * hk)
        k = nq + q
        v = np.concatenate([2 * nq + h * hv + np.arange(hv) for h in self.heads])
        self.channels = np.concatenate([q, k, v])             # qkv rows, conv taps, ring channels
        self.z_rows = np.concatenate([h * hv + np.arange(hv) for h in self.heads])
        self.head_rows = self.heads.copy()                      # beta, alpha, dt_bias, a
        # The local grouped output is the global block [k0*rep*hv, k1*rep*hv).
        self.out0, self.out1 = self.k0 * rep * hv, self.k1 * rep * hv


# Shards of a device image -------------------------------------------------------------------------

def _slice_rows(dt, rows):
    """A DeviceTensor of the given rows (an index array) of `dt`, with dt's B and R."""
    import torch
    from . import ops
    from . import layout as L
    rb = L.row_bytes(dt.cols, dt.kind)
    idx = torch.as_tensor(np.asarray(rows), dtype=torch.long, device=dt.data.device)
    data = dt.data.view(dt.rows, rb).index_select(0, idx).contiguous().view(-1)
    return ops.DeviceTensor.from_packed(data, len(rows), dt.cols, dt.kind, dt.bias, dt.rshift)


class ShardPacked:
    """Row subsets of the segments of a decoder.Packed, back to back (one segmented launch)."""

    def __init__(self, packed, seg_rows):
        import torch
        from . import _lib
        parts, self.entries, self.rows = [], [], []
        for i, rows in enumerate(seg_rows):
            t = _slice_rows(packed.tensor(i), rows)
            parts.append(t.data)
            self.entries.append(_lib.Entry(len(rows), t.cols, t.kind, t.bias, t.rshift))
            self.rows.append(len(rows))
        self.data = torch.cat(parts)
        self.cols, self.kind = packed.cols, packed.kind


class TPWeights:
    """One rank's shard of a decoder.SyntheticWeights (every rank draws the same seeded image and
    keeps its rows; the B/R of each tensor are the full tensor's)."""

    def __init__(self, full, rank, world):
        import torch
        cfg = self.cfg = full.cfg
        self.rank, self.world = rank, world
        E, F, V = cfg.hidden, cfg.ffn, cfg.vocab
        self.e0, self.e1 = span(E, rank, world)
        self.f0, self.f1 = span(F, rank, world)
        self.v0, self.v1 = span(V, rank, world)
        er = np.arange(self.e0, self.e1)
        fr = np.arange(self.f0, self.f1)
        self.emb, self.out_norm, self.rope_freq = full.emb, full.out_norm, full.rope_freq
        self.lm_head = _slice_rows(full.lm_head, np.arange(self.v0, self.v1))
        self.layers = []
        for l, lw in enumerate(full.layers):
            # A K-segmented down projection (ffn wider than one tensor) keeps its segments, each cut
            # to the rank's output rows.
            down = ([_slice_rows(sg, er) for sg in lw["down"]] if isinstance(lw["down"], list)
                    else _slice_rows(lw["down"], er))
            w = {"attn_norm": lw["attn_norm"], "ffn_norm": lw["ffn_norm"],
                 "gate": _slice_rows(lw["gate"], fr), "up": _slice_rows(lw["up"], fr),
                 "down": down, "out": _slice_rows(lw["out"], er)}
            if cfg.layer_type(l) == "d":
                sh = w["shard"] = DeltaNetShard(cfg, rank, world)
                w["in"] = ShardPacked(lw["in"], [sh.channels, sh.z_rows, sh.head_rows, sh.head_rows])
                idx = lambda t, rows: t.index_select(0, torch.as_tensor(rows, device=t.device)).contiguous()
                w["conv_w"] = idx(lw["conv_w"], sh.channels)
                w["ssm_a"] = idx(lw["ssm_a"], sh.heads)
                w["dt_bias"] = idx(lw["dt_bias"], sh.heads)
                w["ssm_norm"] = lw["ssm_norm"]
            else:
                sh = w["shard"] = AttnShard(cfg, rank, world)
                w["in"] = ShardPacked(lw["in"], [sh.q_rows, sh.k_rows, sh.v_rows])
                w["q_norm"], w["k_norm"] = lw["q_norm"], lw["k_norm"]
            self.layers.append(w)


# The tensor-parallel decoder ----------------------------------------------------------------------

def exchange_plan(n_layer):
    """The peer-memory exchanges of one step, in launch order: (op, layer, gather point signalled or
    None, gather point waited on or None).  Gather points: layer l: 4l attention output, 4l+1 x
    after o, 4l+2 act, 4l+3 x after down; 4*n_layer the LM-head keys."""
    plan = []
    for l in range(n_layer):
        plan += [("qkv", l, None, 4 * l - 1 if l else None), ("attn", l, 4 * l, None),
                 ("o", l, 4 * l + 1, 4 * l), ("swiglu", l, 4 * l + 2, 4 * l + 1), ("down", l, 4 * l + 3, 4 * l + 2)]
    plan += [("lm", n_layer - 1, 4 * n_layer, 4 * n_layer - 1), ("token", n_layer - 1, None, 4 * n_layer)]
    return plan


class TPDecoder:
    """Greedy batch-1 decoding of a TPWeights shard; every rank runs the same steps in the same order.
    The exchanges are NCCL all-gathers on `group` captured with the kernels in one CUDA graph, or
    (p2p=True) tagged words that the kernels store into every rank's copy and poll themselves."""

    def __init__(self, weights: TPWeights, group=None, ctx=None, max_pos=4096, p2p=False):
        import torch
        from . import ops
        cfg = self.cfg = weights.cfg
        self.w, self.group = weights, group
        self.ctx = ctx or ops.default_context()
        self.rank, self.world = weights.rank, weights.world
        dev = weights.emb.device
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)
        E, F, N = cfg.hidden, cfg.ffn, self.world
        self.x, self.x_loc = f32(E), f32(E // N)
        self.act, self.act_loc = f32(F), f32(F // N)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.key = torch.zeros(1, dtype=torch.int64, device=dev)
        self.keys = torch.zeros(N, dtype=torch.int64, device=dev)
        self.max_pos = max_pos
        self.kc, self.vc, self.ring, self.state = {}, {}, {}, {}
        a_sh = d_sh = None
        for l, lw in enumerate(weights.layers):
            sh = lw["shard"]
            if cfg.layer_type(l) == "d":
                d_sh = sh
                C = len(sh.channels)
                self.ring[l] = torch.zeros(cfg.dn_conv, C, device=dev)
                self.state[l] = torch.zeros(sh.nv, cfg.dn_hv, cfg.dn_hk, device=dev)
            else:
                a_sh = sh
                self.kc[l] = torch.zeros(max_pos, sh.n_kv, cfg.head_dim, dtype=torch.float16, device=dev)
                self.vc[l] = torch.zeros_like(self.kc[l])
        if a_sh is not None:
            self.attn_shape = ops.attn_shape(a_sh.n_head, a_sh.n_kv, cfg.head_dim, max_pos,
                                             rope_dims=cfg.rope_dims or cfg.head_dim, gated=cfg.attn_gated,
                                             eps=cfg.eps)
            self.q, self.k, self.v = f32(len(a_sh.q_rows)), f32(len(a_sh.k_rows)), f32(len(a_sh.v_rows))
            self.attn_loc = f32(a_sh.n_head * cfg.head_dim)
            self.attn = f32(cfg.n_head * cfg.head_dim)
        if d_sh is not None:
            self.dn_shape = ops.deltanet_shape(d_sh.nk, cfg.dn_hk, d_sh.nv, cfg.dn_hv, cfg.dn_conv, cfg.eps)
            self.qkv, self.z = f32(len(d_sh.channels)), f32(d_sh.nv * cfg.dn_hv)
            self.beta, self.alpha = f32(d_sh.nv), f32(d_sh.nv)
            self.og_loc, self.og = f32(d_sh.nv * cfg.dn_hv), f32(cfg.dn_nv * cfg.dn_hv)
        self.graph = None
        self.p2p = bool(p2p) and self.world > 1 and self._p2p_supported(a_sh)
        if self.p2p:
            self._setup_p2p(a_sh)

    # Exchange over peer memory ------------------------------------------------------------------
    # Instead of an NCCL all-gather after each sharded projection, the producing kernel stores each
    # result into every rank's copy of the vector (peer-mapped symmetric buffers) as one tagged
    # 64-bit word (value bits | tag << 32, tag = step * points + point + 1); the consuming kernel
    # polls its own copy until every word carries the tag it expects.  No fence, no counter, no
    # collective on the path.  Gather points per step: per layer attention output (4l), x after o
    # (4l+1), act (4l+2), x after down (4l+3); then the LM-head keys (4L), exchanged as plain words
    # with a completion counter (one per step).
    def _p2p_supported(self, a_sh):
        """Every layer type and tensor exchanges tagged words (attention of any head dim, DeltaNet,
        K-segmented projections)."""
        return True

    def _setup_p2p(self, a_sh):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        from . import _lib
        cfg, dev = self.cfg, self.tok.device
        gname = (self.group or dist.group.WORLD).group_name
        self._symm = []

        def shared(n, dtype):
            t = symm.empty(n, dtype=dtype, device=dev)
            t.zero_()
            h = symm.rendezvous(t, gname)
            self._symm.append((t, h))
            base = [int(p) for p in h.buffer_ptrs]
            off = t.data_ptr() - base[self.rank]  # the tensor's place inside its symmetric block
            return t, [b + off for b in base]

        E, F, N = cfg.hidden, cfg.ffn, self.world
        types = {cfg.layer_type(l) for l in range(cfg.n_layer)}
        self.n_points = 4 * cfg.n_layer + 1
        self.x_tag, px = shared(E, torch.int64)
        self.attn_tag, pa = shared(cfg.n_head * cfg.head_dim, torch.int64) if "a" in types else (None, None)
        self.og_tag, pg = shared(cfg.dn_nv * cfg.dn_hv, torch.int64) if "d" in types else (None, None)
        self.act_tag, pf = shared(F, torch.int64)
        self.keys, pk = shared(N, torch.int64)
        self.cnt, pc = shared(self.n_points, torch.int32)
        self.step_ctr = torch.zeros(1, dtype=torch.int32, device=dev)
        self.arrive = torch.zeros(self.n_points, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        w, r = self.w, self.rank
        lm_point = 4 * cfg.n_layer

        def xfer(op, l, sig, wt):
            t = _lib.TpXfer()
            t.world, t.rank = N, r
            t.step = self.step_ctr.data_ptr()
            t.tag_points = self.n_points
            if op == "lm":  # the key: a plain word into the other ranks' slots, then their counters
                t.offset = r
                for q in range(N):
                    t.dst[q] = pk[q] if q != r else None
                    t.signal[q] = pc[q] + 4 * lm_point
                t.arrive = self.arrive.data_ptr() + 4 * lm_point
            elif op == "token":
                t.wait = self.cnt.data_ptr() + 4 * lm_point
            elif sig is not None:  # a tagged output into every rank's copy, this rank's included
                sh = w.layers[l]["shard"]
                if op == "attn":  # the mixer's output: attention heads or the DeltaNet grouped block
                    ptrs, t.offset = (pg, sh.out0) if cfg.layer_type(l) == "d" else (pa, sh.head0 * cfg.head_dim)
                else:
                    ptrs, t.offset = {"o": (px, w.e0), "swiglu": (pf, w.f0), "down": (px, w.e0)}[op]
                for q in range(N):
                    t.dst[q] = ptrs[q]
                t.tag_out = sig
            if wt is not None and op != "token":
                t.tag_in = wt
            return t

        self._tp = [dict() for _ in range(cfg.n_layer)]
        for op, l, sig, wt in exchange_plan(cfg.n_layer):
            t = xfer(op, l, sig, wt) if (sig is not None or wt is not None) else None
            if op == "lm":
                self._tp_lm = t
            elif op == "token":
                self._tp_tok = t
            else:
                self._tp[l][op] = t

    def _gather(self, out, inp):
        import torch.distributed as dist
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_gather_into_tensor(out, inp, group=self.group)

    def set_states(self, seed=0):
        """The global DeltaNet states ~N(0,1)/sqrt(hk) of Decoder.set_states, this rank's heads."""
        import math
        import torch
        g = torch.Generator(device=self.tok.device)
        g.manual_seed(seed)
        cfg = self.cfg
        for l, t in sorted(self.state.items()):
            full = torch.randn((cfg.dn_nv, cfg.dn_hv, cfg.dn_hk), generator=g, device=t.device) / math.sqrt(cfg.dn_hk)
            heads = torch.as_tensor(self.w.layers[l]["shard"].heads, device=t.device)
            t.copy_(full.index_select(0, heads))

    def fill_context(self, n, seed=0):
        """Synthetic context of n positions (random fp16 K/V rows of this rank's heads), position n.
        Seeded by the rank's first kv head, so ranks that replicate a kv head hold the same cache."""
        import torch
        g = torch.Generator(device=self.tok.device)
        a_sh = next((lw["shard"] for lw in self.w.layers if isinstance(lw["shard"], AttnShard)), None)
        g.manual_seed(seed + (a_sh.kv0 if a_sh is not None else self.rank))
        for l in self.kc:
            self.kc[l][:n] = torch.randn(self.kc[l][:n].shape, generator=g, device=self.tok.device).half()
            self.vc[l][:n] = torch.randn(self.vc[l][:n].shape, generator=g, device=self.tok.device).half()
        self.pos.fill_(n)

    def enqueue_step(self):
        """One token on every rank: reads self.tok and self.pos, writes the next token (the same on
        every rank) and advances the position."""
        if self.p2p:
            return self._enqueue_step_p2p()
        from . import ops
        cfg, w, ctx = self.cfg, self.w, self.ctx
        xr = self.x[w.e0:w.e1]  # this rank's rows of the residual stream
        ops.embed_lookup(ctx, w.emb, self.tok, self.x)
        for l, lw in enumerate(w.layers):
            p = lw["in"]
            if cfg.layer_type(l) == "d":
                ops.matvec_f_multi(ctx, p.entries, p.data, self.x, [self.qkv, self.z, self.beta, self.alpha],
                                   norm_w=lw["attn_norm"], eps=cfg.eps)
                ops.deltanet_step(ctx, self.dn_shape, self.qkv, self.z, self.beta, self.alpha, lw["dt_bias"],
                                  lw["ssm_a"], lw["conv_w"], lw["ssm_norm"], self.ring[l], self.state[l], self.pos,
                                  self.og_loc)
                self._gather(self.og, self.og_loc)
                ops.matvec_f(ctx, lw["out"], self.og, y=self.x_loc, resid=xr)
            else:
                ops.matvec_f_multi(ctx, p.entries, p.data, self.x, [self.q, self.k, self.v], norm_w=lw["attn_norm"],
                                   eps=cfg.eps)
                ops.attn_decode(ctx, self.attn_shape, self.q, self.k, self.v, lw["q_norm"], lw["k_norm"], w.rope_freq,
                                self.kc[l], self.vc[l], self.pos, self.attn_loc)
                self._gather(self.attn, self.attn_loc)
                ops.matvec_f(ctx, lw["out"], self.attn, y=self.x_loc, resid=xr)
            self._gather(self.x, self.x_loc)
            ops.matvec_swiglu(ctx, lw["gate"], lw["up"], self.x, act=self.act_loc, norm_w=lw["ffn_norm"], eps=cfg.eps)
            self._gather(self.act, self.act_loc)
            if isinstance(lw["down"], list):
                ops.matvec_f_kseg(ctx, lw["down"], self.act, y=self.x_loc, resid=xr)
            else:
                ops.matvec_f(ctx, lw["down"], self.act, y=self.x_loc, resid=xr)
            self._gather(self.x, self.x_loc)
        ops.lmhead_argmax_key(ctx, w.lm_head, self.x, self.key, row_offset=w.v0, norm_w=w.out_norm, eps=cfg.eps)
        self._gather(self.keys, self.key)
        ops.argmax_token(ctx, self.keys, self.tok)
        ops.advance_position(ctx, self.pos)

    def _enqueue_step_p2p(self):
        from . import ops
        cfg, w, ctx = self.cfg, self.w, self.ctx
        x_loc = self.x_loc  # this rank's rows of the residual stream (local floats)
        ops.embed_lookup(ctx, w.emb, self.tok, self.x)
        for l, lw in enumerate(w.layers):
            t = self._tp[l]
            p = lw["in"]
            xin = self.x if l == 0 else self.x_tag  # the embedding (local floats), then the tagged x
            if cfg.layer_type(l) == "d":
                ops.matvec_f_multi(ctx, p.entries, p.data, xin, [self.qkv, self.z, self.beta, self.alpha],
                                   norm_w=lw["attn_norm"], eps=cfg.eps, tp=t["qkv"])
                ops.deltanet_step(ctx, self.dn_shape, self.qkv, self.z, self.beta, self.alpha, lw["dt_bias"],
                                  lw["ssm_a"], lw["conv_w"], lw["ssm_norm"], self.ring[l], self.state[l], self.pos,
                                  self.og_loc, tp=t["attn"])
                mix = self.og_tag
            else:
                ops.matvec_f_multi(ctx, p.entries, p.data, xin, [self.q, self.k, self.v], norm_w=lw["attn_norm"],
                                   eps=cfg.eps, tp=t["qkv"])
                ops.attn_decode(ctx, self.attn_shape, self.q, self.k, self.v, lw["q_norm"], lw["k_norm"],
                                w.rope_freq, self.kc[l], self.vc[l], self.pos, self.attn_loc, tp=t["attn"])
                mix = self.attn_tag
            ops.matvec_f(ctx, lw["out"], mix, y=x_loc, resid=self.x[w.e0:w.e1] if l == 0 else x_loc, tp=t["o"])
            ops.matvec_swiglu(ctx, lw["gate"], lw["up"], self.x_tag, act=self.act_loc, norm_w=lw["ffn_norm"],
                              eps=cfg.eps, tp=t["swiglu"])
            if isinstance(lw["down"], list):
                ops.matvec_f_kseg(ctx, lw["down"], self.act_tag, y=x_loc, resid=x_loc, tp=t["down"])
            else:
                ops.matvec_f(ctx, lw["down"], self.act_tag, y=x_loc, resid=x_loc, tp=t["down"])
        ops.lmhead_argmax_key(ctx, w.lm_head, self.x_tag, self.keys[self.rank:self.rank + 1], row_offset=w.v0,
                              norm_w=w.out_norm, eps=cfg.eps, tp=self._tp_lm)
        ops.argmax_token(ctx, self.keys, self.tok, tp=self._tp_tok)
        ops.advance_position(ctx, self.pos)
        ops.advance_position(ctx, self.step_ctr)

    def collectives_per_step(self):
        """NCCL collectives per step (0 when the exchanges go over peer memory)."""
        if self.p2p:
            return 0
        return 4 * self.cfg.n_layer + 1

    def _mutable(self):
        extra = ([self.cnt, self.step_ctr, self.arrive, self.x_tag, self.act_tag] +
                 [t for t in (self.attn_tag, self.og_tag) if t is not None]) if self.p2p else []
        return [self.tok, self.pos] + list(self.kc.values()) + list(self.vc.values()) + list(self.ring.values()) + \
            list(self.state.values()) + extra

    def capture(self):
        """One step as a CUDA graph on every rank (NCCL collectives captured with the kernels)."""
        import torch
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
        if self.p2p:  # every rank's counters are restored before any rank signals again
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self.enqueue_step()
        torch.cuda.synchronize()
        return self.graph

    def release(self):
        """Drop the captured graph (it holds NCCL work: release it before destroying the group)."""
        self.graph = None

    def step(self, token=None):
        if token is not None:
            self.tok.fill_(int(token))
        if self.graph is not None:
            self.graph.replay()
        else:
            self.enqueue_step()

    def generate(self, prompt, n_new):
        """Greedy decode as decoder.Decoder.generate (mirror.py:1036-1044), the same on every rank."""
        import torch
        for t in prompt:
            self.step(t)
        out = torch.empty(n_new, dtype=torch.int32, device=self.tok.device)
        for i in range(n_new):
            out[i:i + 1].copy_(self.tok)
            if i + 1 < n_new:
                self.step()
        self.ctx.raise_on_error()
        return out.cpu().tolist()
