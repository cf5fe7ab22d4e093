"""Runtime hybrid target: packed per-rank weights, paged KV, GDN state slots, and the three
forward modes the speculative runtime needs.

* ``prefill`` - committed, chunked (``RuntimeConfig.prefill_chunk`` rows per chunk, GDN state
  and conv window carried across chunks); the reference's chunk-outer prefill
  (``scripts/ci/fixtures/qwen36_model.py:2261,2482-2520``).
* ``verify`` - uncommitted forward of a block of rows for one or more sequences (packed
  multi-user verify, ``scripts/ci/packed_verifier.py:1-12``).  K/V rows are written past the
  committed frontier; GDN state and conv windows are read, never written.  The in-projection
  rows of every GDN layer are kept for ``commit``.
* ``commit`` - publish the accepted prefix: GDN state and window advance by replaying the kept
  rows through the same recurrence, so the committed state is bit-identical to single-row decode
  (the reference's commit-only GDN, ``docs/dflash-commit-only-gdn-2026-09-09.md``, with the
  retained histories replaced by a replay of the tiny projected rows).

Tensor parallelism (``tp_widths``): column-parallel in-projections over heads, row-parallel
out-projections whose fp32 partials are summed across ranks, replicated residual, vocab-parallel
LM head with a cross-rank (value, index) argmax.  Layout per rank:

* GDN in-projection rows ``[q | k | v | z | b | a]`` of the rank's heads (the reference's fused
  ``qkvzab``, ``graft/gdn/tp.py:77-103``), conv taps ``[C_local, K]``.
* attention in-projection rows ``[q | gate | k | v]`` (``graft/attention/tp.py:177``).
* MLP gate/up interleaved in blocks of ``GU_BLOCK`` rows ``[gate | up]`` so a GEMM tile holds
  matching gate and up features and the SwiGLU can run in its epilogue.
"""
from __future__ import annotations

import os

from dataclasses import dataclass, field

import torch

from ..config import FULL, LINEAR, ModelConfig, RuntimeConfig, tp_widths
from ..ops import torch_ref as R

GU_BLOCK = 64


# ------------------------------------------------------------------------------------ packing
def _rows(t, start, count):
    return t[start:start + count]


def pack_gdn(src, i, cfg: ModelConfig, tp, r, device, dtype):
    p = f"model.layers.{i}.linear_attn."
    nk, nv, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, \
        cfg.linear_value_head_dim
    nkl, nvl = nk // tp, nv // tp
    kd = nk * dk
    qkv = src.get(p + "in_proj_qkv.weight", device=device, dtype=dtype)
    z = src.get(p + "in_proj_z.weight", device=device, dtype=dtype)
    b = src.get(p + "in_proj_b.weight", device=device, dtype=dtype)
    a = src.get(p + "in_proj_a.weight", device=device, dtype=dtype)
    q_l = _rows(qkv, r * nkl * dk, nkl * dk)
    k_l = _rows(qkv, kd + r * nkl * dk, nkl * dk)
    v_l = _rows(qkv, 2 * kd + r * nvl * dv, nvl * dv)
    parts = [q_l, k_l, v_l, _rows(z, r * nvl * dv, nvl * dv), _rows(b, r * nvl, nvl), _rows(a, r * nvl, nvl)]
    pad = -sum(t.shape[0] for t in parts) % 8       # projection rows stay 16-byte aligned (e.g. 2060 at TP8)
    if pad:
        parts.append(q_l.new_zeros(pad, q_l.shape[1]))
    w_in = torch.cat(parts, 0).contiguous()
    conv = src.get(p + "conv1d.weight", device=device, dtype=torch.float32)
    conv = conv.reshape(conv.shape[0], -1)
    conv_l = torch.cat([_rows(conv, r * nkl * dk, nkl * dk), _rows(conv, kd + r * nkl * dk, nkl * dk),
                        _rows(conv, 2 * kd + r * nvl * dv, nvl * dv)], 0).contiguous()
    out = src.get(p + "out_proj.weight", device=device, dtype=dtype)
    return dict(
        kind=LINEAR,
        w_in=w_in,
        conv_w=conv_l,
        A_log=_rows(src.get(p + "A_log", device=device, dtype=torch.float32).float(), r * nvl, nvl).contiguous(),
        dt_bias=_rows(src.get(p + "dt_bias", device=device, dtype=torch.float32).float(), r * nvl, nvl).contiguous(),
        norm_w=src.get(p + "norm.weight", device=device, dtype=torch.float32).float().contiguous(),
        w_out=out[:, r * nvl * dv:(r + 1) * nvl * dv].contiguous(),
        dims=(nkl, nvl, dk, dv),
    )


def pack_attn(src, i, cfg: ModelConfig, tp, r, device, dtype, prefix=None):
    p = (prefix or f"model.layers.{i}.") + "self_attn."
    H, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    w = tp_widths(cfg, tp)
    hl = w["n_heads"]
    qp = src.get(p + "q_proj.weight", device=device, dtype=dtype).view(H, 2, D, -1)
    q_l = qp[r * hl:(r + 1) * hl, 0].reshape(hl * D, -1)
    g_l = qp[r * hl:(r + 1) * hl, 1].reshape(hl * D, -1)
    kw = src.get(p + "k_proj.weight", device=device, dtype=dtype)
    vw = src.get(p + "v_proj.weight", device=device, dtype=dtype)
    if w["kv_replication"]:
        kvh = r * Hkv // tp
        k_l, v_l = _rows(kw, kvh * D, D), _rows(vw, kvh * D, D)
    else:
        nkl = w["n_kv"]
        k_l, v_l = _rows(kw, r * nkl * D, nkl * D), _rows(vw, r * nkl * D, nkl * D)
    o = src.get(p + "o_proj.weight", device=device, dtype=dtype)
    one = lambda n: (1.0 + src.get(p + n, device=device, dtype=torch.float32).float()).contiguous()
    return dict(
        kind=FULL,
        w_in=torch.cat([q_l, g_l, k_l, v_l], 0).contiguous(),
        qn=one("q_norm.weight"), kn=one("k_norm.weight"),
        w_out=o[:, r * hl * D:(r + 1) * hl * D].contiguous(),
        dims=(hl, w["n_kv"], D),
    )


def pack_mlp(src, i, cfg: ModelConfig, tp, r, device, dtype, prefix=None):
    p = (prefix or f"model.layers.{i}.") + "mlp."
    il = cfg.intermediate_size // tp
    if il % GU_BLOCK:
        raise ValueError(f"per-rank intermediate {il} must be a multiple of {GU_BLOCK}")
    g = _rows(src.get(p + "gate_proj.weight", device=device, dtype=dtype), r * il, il)
    u = _rows(src.get(p + "up_proj.weight", device=device, dtype=dtype), r * il, il)
    H = g.shape[1]
    gu = torch.stack([g.reshape(il // GU_BLOCK, GU_BLOCK, H), u.reshape(il // GU_BLOCK, GU_BLOCK, H)], 1)
    d = src.get(p + "down_proj.weight", device=device, dtype=dtype)
    return dict(w_gu=gu.reshape(2 * il, H).contiguous(), w_down=d[:, r * il:(r + 1) * il].contiguous())


# ------------------------------------------------------------------------------------ state
class BlockAllocator:
    """Reference-counted free-list allocator of fixed-size KV blocks.  A block is shared by every
    sequence and prefix checkpoint that holds it and returns to the free list when the last holder
    releases it."""

    def __init__(self, num_blocks: int):
        self.free = list(range(num_blocks - 1, -1, -1))
        self.refs = [0] * num_blocks
        self.num_blocks = num_blocks

    def alloc(self, n: int) -> list:
        if n > len(self.free):
            raise MemoryError(f"KV pool exhausted: need {n} blocks, {len(self.free)} free")
        out = [self.free.pop() for _ in range(n)]
        for b in out:
            self.refs[b] = 1
        return out

    def incref(self, blocks):
        for b in blocks:
            if self.refs[b] <= 0:
                raise ValueError(f"block {b} is not allocated")
            self.refs[b] += 1

    def release(self, blocks):
        for b in reversed(list(blocks)):
            if self.refs[b] <= 0:
                raise ValueError(f"double release of block {b}")
            self.refs[b] -= 1
            if self.refs[b] == 0:
                self.free.append(b)

    @property
    def num_free(self):
        return len(self.free)


@dataclass
class SeqState:
    slot: int
    block_table: torch.Tensor          # [max_blocks] int32 (device)
    blocks: list = field(default_factory=list)
    pos: int = 0                       # committed tokens
    verify_rows: tuple | None = None   # (row offset, rows) of this sequence in the last verify
    closed: bool = False


class HybridTarget:
    def __init__(self, cfg: ModelConfig, src, rt: RuntimeConfig | None = None, *, device="cpu",
                 dtype=torch.float32, ops=None, comm=None, max_slots: int = 1, kv_blocks: int | None = None,
                 max_verify_rows: int = 32, kv_dtype=None):
        from ..ops import TorchOps
        from ..parallel.comm import NullComm
        self.cfg = cfg
        self.rt = rt or RuntimeConfig()
        self.device = torch.device(device)
        self.dtype = dtype
        self.ops = ops or TorchOps()
        self.comm = comm or NullComm()
        # pushed all-reduce: out-projection GEMMs push their partial tiles to every rank; the next
        # RMSNorm of the residual completes the reduction (``_pending`` = (residual, "push", slot), or
        # (residual, "rs", completion-flag target) for the fused prefill all-reduce)
        self.fused_ar = bool(getattr(self.comm, "fused", False)) and hasattr(ops, "linear_push")
        # single rank: out-projections of <= 64 rows leave their split-K slices for the next norm
        # (``_pending`` = (residual, "split", slice count)); Q38_DEFER_SPLITK=0 keeps the in-GEMM fix-up
        self.defer_splits = hasattr(self.ops, "linear_split") and os.environ.get("Q38_DEFER_SPLITK", "1") != "0"
        self._pending = None
        # rows one verify may pack and stay on the batch-invariant kernels (None: no limit)
        self.max_pack_rows = getattr(self.ops, "max_pack_rows", None)
        tp, r = self.comm.world, self.comm.rank
        self.tp, self.rank = tp, r
        self.widths = tp_widths(cfg, tp)
        self.eps = cfg.rms_norm_eps
        f32 = dict(device=self.device, dtype=torch.float32)

        # ---- weights
        self.embed = src.get("model.embed_tokens.weight", device=self.device, dtype=dtype).contiguous()
        head = self.embed if cfg.tie_word_embeddings else src.get("lm_head.weight", device=self.device, dtype=dtype)
        vl = self.widths["vocab"]
        self.vocab_offset = r * vl
        self.lm_head = self.ops.prepare_weight(head[r * vl:(r + 1) * vl].contiguous())
        del head
        self.final_norm = (1.0 + src.get("model.norm.weight", **f32).float()).contiguous()
        self.layers = []
        for i, t in enumerate(cfg.layer_types):
            pfx = f"model.layers.{i}."
            L = pack_gdn(src, i, cfg, tp, r, self.device, dtype) if t == LINEAR else \
                pack_attn(src, i, cfg, tp, r, self.device, dtype)
            L.update(pack_mlp(src, i, cfg, tp, r, self.device, dtype))
            L["in_norm"] = (1.0 + src.get(pfx + "input_layernorm.weight", **f32).float()).contiguous()
            L["post_norm"] = (1.0 + src.get(pfx + "post_attention_layernorm.weight", **f32).float()).contiguous()
            for key in ("w_in", "w_out", "w_gu", "w_down"):
                L[key] = self.ops.prepare_weight(L[key])
            self.layers.append(L)
        self.gdn_index = {i: j for j, i in enumerate(cfg.linear_layers)}
        self.attn_index = {i: j for j, i in enumerate(cfg.full_layers)}
        # per-layer GDN parameters stacked [Lg, ...] so one launch can commit every layer;
        # each layer's dict entries become views into the stacks
        if cfg.linear_layers:
            for key in ("conv_w", "A_log", "dt_bias", "norm_w"):
                stack = torch.stack([self.layers[i][key] for i in cfg.linear_layers]).contiguous()
                setattr(self, "gdn_" + key, stack)
                for j, i in enumerate(cfg.linear_layers):
                    self.layers[i][key] = stack[j]

        # ---- RoPE inverse frequencies (partial rotary, half-split)
        rd = cfg.rope_dim
        self.inv_freq = (1.0 / (cfg.rope_theta ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))).to(self.device)

        # ---- GDN state slots
        g = self.layers[cfg.linear_layers[0]] if cfg.linear_layers else None
        self.max_slots = max_slots
        if g is not None:
            nkl, nvl, dk, dv = g["dims"]
            C = 2 * nkl * dk + nvl * dv
            K = cfg.linear_conv_kernel_dim
            Lg = len(cfg.linear_layers)
            self.rec = torch.zeros(max_slots, Lg, nvl, dk, dv, **f32)
            self.conv = torch.zeros(max_slots, Lg, K - 1, C, device=self.device, dtype=dtype)
            self.gdn_in_width = g["w_in"].shape[0]
            # rows of the last verify, kept for commit
            self.gdn_stash = torch.zeros(Lg, max_verify_rows, self.gdn_in_width, device=self.device, dtype=dtype)
        self.max_verify_rows = max_verify_rows
        self.free_slots = list(range(max_slots - 1, -1, -1))

        # ---- paged KV
        bs = self.rt.kv_block_size
        self.block_size = bs
        self.max_blocks_per_seq = -(-self.rt.max_context // bs) + 1
        if kv_blocks is None:
            kv_blocks = self.max_blocks_per_seq * max_slots
        La = len(cfg.full_layers)
        hkv, D = self.widths["n_kv"], cfg.head_dim
        kvd = kv_dtype or dtype
        self.kcache = torch.zeros(max(La, 1), kv_blocks, bs, hkv, D, device=self.device, dtype=kvd)
        self.vcache = torch.zeros(max(La, 1), kv_blocks, bs, hkv, D, device=self.device, dtype=kvd)
        self.allocator = BlockAllocator(kv_blocks)
        # per-slot block tables at fixed addresses (captured graphs reference them)
        self.block_tables = torch.zeros(max_slots, self.max_blocks_per_seq, dtype=torch.int32, device=self.device)
        self.use_graphs = bool(self.rt.use_cuda_graphs) and self.device.type == "cuda"
        self._graphs = {}
        self._graph_pool = None

    # ------------------------------------------------------------------ sequences
    def new_sequence(self) -> SeqState:
        if not self.free_slots:
            raise MemoryError("no free GDN state slot")
        slot = self.free_slots.pop()
        if hasattr(self, "rec"):
            self.rec[slot].zero_()
            self.conv[slot].zero_()
        bt = self.block_tables[slot]
        bt.zero_()
        return SeqState(slot=slot, block_table=bt)

    def release(self, seq: SeqState):
        if seq.closed:
            return
        self.allocator.release(seq.blocks)
        seq.blocks = []
        self.free_slots.append(seq.slot)
        seq.closed = True

    def reserve(self, seq: SeqState, upto: int):
        """Make sure KV blocks cover positions [0, upto)."""
        need = -(-upto // self.block_size)
        if need > self.max_blocks_per_seq:
            raise ValueError(f"context {upto} exceeds max_context {self.rt.max_context}")
        if need > len(seq.blocks):
            new = self.allocator.alloc(need - len(seq.blocks))
            seq.blocks.extend(new)
            seq.block_table[len(seq.blocks) - len(new):len(seq.blocks)] = torch.tensor(
                new, dtype=torch.int32, device=self.device)

    def positions(self, start: int, n: int):
        return torch.arange(start, start + n, device=self.device, dtype=torch.int32)

    # ------------------------------------------------------------------ blocks
    def _row_parallel(self, h, w, x):
        """x += h @ w^T summed over ranks (row-parallel out-projection + residual add)."""
        if self.tp == 1:
            self.local_row_parallel(h, w, x)
        elif self.fused_ar and self.comm.fused_fits(*x.shape):
            self.push_row_parallel(h, w, x)
        elif getattr(self.comm, "prefill_fits", None) is not None and self.comm.prefill_fits(x):
            # prefill chunk: reduce-scatter GEMM + owner reduce + multicast broadcast, completed by
            # the next norm / settle of x
            self.settle(x)
            self._pending = (x, "rs", self.comm.prefill_push(self.ops, h, self.ops.prepare_weight(w), x))
        elif hasattr(self.comm, "slot_out") and self.comm.fits(*x.shape):
            slot, part = self.comm.slot_out(*x.shape)          # GEMM writes into peer memory
            self.ops.linear(h, w, out=part)
            self.comm.reduce_slot_add(slot, x)
        else:
            part = self.ops.linear(h, w, out_dtype=torch.float32)
            self.comm.all_reduce_(part)
            x += part

    def local_row_parallel(self, h, w, x):
        """x += h @ w^T on one rank; for <= 32 rows the split-K slices are added by the next
        ``norm`` / ``settle`` of x (the drafters use it too)."""
        if self.defer_splits and x.shape[0] <= self.ops.max_pack_rows:
            self.settle(x)
            S = self.ops.linear_split(h, w, x)
            if S > 1:
                self._pending = (x, "split", S)
        else:
            self.ops.linear_residual(h, w, x)

    def norm(self, x, w, eps=None):
        """RMSNorm of the residual ``x``; completes a pending pushed all-reduce into ``x`` first
        (in the same kernel)."""
        eps = self.eps if eps is None else eps
        if self._pending is not None and self._pending[0] is x:
            _, kind, val = self._pending
            self._pending = None
            if kind == "rs":
                return self.comm.prefill_norm(self.ops, x, w, eps, val)
            if kind == "split":
                return self.ops.rms_norm_split(x, w, eps, self.dtype, val)
            return self.ops.rms_norm_ar(x, w, eps, self.dtype, self.comm, val)
        return self.ops.rms_norm(x, w, eps, self.dtype)

    def push_row_parallel(self, h, w, x):
        """Pushed all-reduce of a row-parallel out-projection into the residual ``x`` (any
        model's residual: the drafters use it too); completed by the next ``norm`` / ``settle``."""
        self.settle(x)
        self._pending = (x, "push", self.ops.linear_push(h, w, self.comm))

    def settle(self, x=None):
        """Complete a pending pushed all-reduce without a norm (before ``x`` is read raw)."""
        if self._pending is not None and (x is None or self._pending[0] is x):
            px, kind, val = self._pending
            self._pending = None
            if kind == "rs":
                self.comm.prefill_wait(self.ops, val)
            elif kind == "split":
                self.ops.rms_norm_split(px, None, self.eps, self.dtype, val)
            else:
                self.ops.rms_norm_ar(px, None, self.eps, self.dtype, self.comm, val)

    def _mlp(self, L, x):
        h = self.norm(x, L["post_norm"])
        gu = self.ops.linear_swiglu(h, L["w_gu"], GU_BLOCK)
        self._row_parallel(gu, L["w_down"], x)

    def _head(self, x_rows, sampling=None):
        hn = self.norm(x_rows, self.final_norm)
        val, idx = (self.ops.lm_head_argmax(hn, self.lm_head, self.vocab_offset, sampling) if sampling is not None
                    else self.ops.lm_head_argmax(hn, self.lm_head, self.vocab_offset))
        return self.comm.argmax_reduce(val, idx) if self.tp > 1 else idx

    def _tap_buffer(self, rows, taps):
        if not taps:
            return None
        return torch.empty(rows, len(taps), self.cfg.hidden_size, device=self.device, dtype=self.dtype)

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, seq: SeqState, tokens: torch.Tensor, taps=(), return_logits_row=False, sampling=None):
        """Committed prefill of ``tokens`` [S] from ``seq.pos``.  Returns (next token [1] int64,
        tap features [S, len(taps)*H] or None)."""
        S = tokens.shape[0]
        self.reserve(seq, seq.pos + S)
        feats = self._tap_buffer(S, taps)
        tap_pos = {t: j for j, t in enumerate(taps)}
        chunk = self.rt.prefill_chunk
        nxt = None
        for c0 in range(0, S, chunk):
            c1 = min(S, c0 + chunk)
            tok = tokens[c0:c1]
            pos0 = seq.pos
            xbuf = self.comm.prefill_x(c1 - c0) if hasattr(self.comm, "prefill_x") else None
            if xbuf is not None:          # the fused prefill all-reduce's symmetric residual
                x = self.ops.embedding(tok, self.embed, out=xbuf)
            else:
                x = self.ops.embedding(tok, self.embed).float()
            positions = self.positions(pos0, tok.shape[0])
            for i, L in enumerate(self.layers):
                h = self.norm(x, L["in_norm"])
                proj = self.ops.linear(h, L["w_in"])
                if L["kind"] == LINEAR:
                    j = self.gdn_index[i]
                    o = self.ops.gdn_prefill(proj, self.conv[seq.slot, j], self.rec[seq.slot, j], L["conv_w"],
                                             L["A_log"], L["dt_bias"], L["norm_w"], self.eps, L["dims"],
                                             self.rt.gdn_chunk, self.dtype)
                else:
                    j = self.attn_index[i]
                    q, gate = self.ops.attn_prep(proj, L["qn"], L["kn"], self.inv_freq, 1.0, self.cfg.rope_dim,
                                                 L["dims"], self.eps, positions, self.kcache[j], self.vcache[j],
                                                 seq.block_table, self.block_size)
                    o = self.ops.attn_prefill(q, gate, self.kcache[j], self.vcache[j], seq.block_table, positions,
                                              self.block_size, self.dtype)
                self._row_parallel(o, L["w_out"], x)
                self._mlp(L, x)
                if i in tap_pos:
                    self.settle(x)
                    feats[c0:c1, tap_pos[i]] = x.to(self.dtype)
            seq.pos += tok.shape[0]
            self.settle(x)                # the next chunk reuses the residual buffer
            if c1 == S:
                nxt = self._head(x[-1:], sampling)
        return nxt, (feats.reshape(S, -1) if feats is not None else None)

    # ------------------------------------------------------------------ verify / commit
    @torch.no_grad()
    def verify(self, batch, taps=(), sampling=None):
        """Uncommitted forward (CUDA-graph replay for a single greedy sequence when enabled).
        ``sampling`` = (scale [rows] fp32, key [rows] int64): rows with scale = 1/temperature > 0
        return Gumbel-max samples instead of argmax tokens."""
        if self.use_graphs and len(batch) == 1 and sampling is None:
            return self._verify_graphed(batch[0][0], batch[0][1], tuple(taps))
        return self._verify_eager(batch, taps, sampling=sampling)

    def _verify_graphed(self, seq: SeqState, tokens: torch.Tensor, taps: tuple):
        T = int(tokens.shape[0])
        if T > self.max_verify_rows:
            raise ValueError(f"{T} verify rows exceed max_verify_rows={self.max_verify_rows}")
        self.reserve(seq, seq.pos + T)
        key = (seq.slot, T, taps)
        g = self._graphs.get(key)
        if g is None:
            g = self._capture_verify(seq, T, taps)
            self._graphs[key] = g
        g["tokens"].copy_(tokens, non_blocking=True)
        g["pos_host"].copy_(torch.arange(seq.pos, seq.pos + T, dtype=torch.int32))
        g["positions"].copy_(g["pos_host"], non_blocking=True)
        seq.verify_rows = (0, T)
        g["graph"].replay()
        if hasattr(self.ops, "launches"):
            self.ops.launches += g["launches"]
        return g["pred"], g["feats"]

    def _capture_verify(self, seq: SeqState, T: int, taps: tuple):
        dev = self.device
        tokens = torch.zeros(T, dtype=torch.long, device=dev)
        positions = torch.arange(seq.pos, seq.pos + T, dtype=torch.int32, device=dev)
        pos_host = torch.zeros(T, dtype=torch.int32).pin_memory()
        saved = seq.pos, seq.verify_rows
        # eager warm-up on the static buffers (kernel attributes, tensor-map caches)
        self._verify_eager([(seq, tokens)], taps, positions=positions)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        l0 = getattr(self.ops, "launches", 0)
        if hasattr(self.comm, "begin_capture"):
            self.comm.begin_capture()
        with torch.cuda.graph(graph):
            pred, feats = self._verify_eager([(seq, tokens)], taps, positions=positions)
        launches = getattr(self.ops, "launches", 0) - l0
        seq.pos, seq.verify_rows = saved
        return dict(graph=graph, tokens=tokens, positions=positions, pos_host=pos_host, pred=pred, feats=feats,
                    launches=launches)

    def release_graphs(self):
        """Drop captured graphs (they may hold NCCL work: release before destroying the process
        group, or the exit waits on them)."""
        self._graphs.clear()
        self._graph_pool = None

    def _pool(self):
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        return self._graph_pool

    def _verify_eager(self, batch, taps=(), positions=None, sampling=None):
        """Uncommitted forward.  ``batch``: list of (SeqState, tokens [T_s]) with the tokens at
        positions ``seq.pos ..``.  Returns (argmax [sum T_s] int64, taps [sum T_s, n*H] or None)."""
        rows = sum(int(t.shape[0]) for _, t in batch)
        if rows > self.max_verify_rows:
            raise ValueError(f"{rows} verify rows exceed max_verify_rows={self.max_verify_rows}")
        off = 0
        for seq, t in batch:
            self.reserve(seq, seq.pos + t.shape[0])
            seq.verify_rows = (off, int(t.shape[0]))
            off += int(t.shape[0])
        tokens = torch.cat([t for _, t in batch]) if len(batch) > 1 else batch[0][1]
        if positions is None:
            positions = torch.cat([self.positions(s.pos, t.shape[0]) for s, t in batch]) if len(batch) > 1 else \
                self.positions(batch[0][0].pos, batch[0][1].shape[0])
        feats = self._tap_buffer(rows, taps)
        tap_pos = {t: j for j, t in enumerate(taps)}
        x = self.ops.embedding(tokens, self.embed).float()
        for i, L in enumerate(self.layers):
            h = self.norm(x, L["in_norm"])
            outs = []
            if L["kind"] == LINEAR:
                j = self.gdn_index[i]
                proj = self.ops.linear(h, L["w_in"], out=self.gdn_stash[j, :rows])   # kept for commit
                for seq, t in batch:
                    o0, n = seq.verify_rows
                    outs.append(self.ops.gdn_verify(proj[o0:o0 + n], self.conv[seq.slot, j], self.rec[seq.slot, j],
                                                    L["conv_w"], L["A_log"], L["dt_bias"], L["norm_w"], self.eps,
                                                    L["dims"], self.dtype))
            else:
                j = self.attn_index[i]
                proj = self.ops.linear(h, L["w_in"])
                for seq, t in batch:
                    o0, n = seq.verify_rows
                    pr = positions[o0:o0 + n]
                    q, gate = self.ops.attn_prep(proj[o0:o0 + n], L["qn"], L["kn"], self.inv_freq, 1.0,
                                                 self.cfg.rope_dim, L["dims"], self.eps, pr, self.kcache[j],
                                                 self.vcache[j], seq.block_table, self.block_size)
                    outs.append(self.ops.attn_decode(q, gate, self.kcache[j], self.vcache[j], seq.block_table,
                                                     pr, self.block_size, self.dtype))
            o = torch.cat(outs, 0) if len(outs) > 1 else outs[0]
            self._row_parallel(o, L["w_out"], x)
            self._mlp(L, x)
            if i in tap_pos:
                self.settle(x)
                feats[:, tap_pos[i]] = x.to(self.dtype)
        pred = self._head(x, sampling)
        return pred, (feats.reshape(rows, -1) if feats is not None else None)

    @torch.no_grad()
    def commit(self, seq: SeqState, n: int):
        """Publish the first ``n`` rows of ``seq``'s last verify."""
        if seq.verify_rows is None:
            raise RuntimeError("commit without a pending verify")
        o0, rows = seq.verify_rows
        if not 0 <= n <= rows:
            raise ValueError(f"commit of {n} rows outside the verified block of {rows}")
        self.commit_device(seq.slot, o0, rows, n)
        seq.pos += n
        seq.verify_rows = None

    def commit_device(self, slot: int, o0: int, rows: int, n: int):
        """The device half of ``commit``: replay the first ``n`` kept GDN rows of the verify block
        at stash rows o0..o0+rows into ``slot``'s state and conv windows (capturable)."""
        if self.cfg.linear_layers and n > 0:
            dims = self.layers[self.cfg.linear_layers[0]]["dims"]
            self.ops.gdn_commit_layers(self.gdn_stash[:, o0:o0 + rows], n, self.conv[slot], self.rec[slot],
                                       self.gdn_conv_w, self.gdn_A_log, self.gdn_dt_bias, dims)

    def abort(self, seq: SeqState):
        """Drop the pending verify: nothing was committed, K/V rows past the frontier are stale."""
        seq.verify_rows = None

    @torch.no_grad()
    def decode(self, seq: SeqState, token: torch.Tensor, taps=()):
        """Plain greedy step = one-row verify + commit of that row (shares every kernel with verify)."""
        pred, feats = self.verify([(seq, token.reshape(1))], taps)
        self.commit(seq, 1)
        return pred, feats

    # ------------------------------------------------------------------ snapshots
    def snapshot(self, seq: SeqState) -> dict:
        """Copy of the sequence's recurrent state (GDN state + conv windows) and length; K/V
        blocks are append-only below ``pos`` and are shared, not copied."""
        snap = {"pos": seq.pos}
        if hasattr(self, "rec"):
            snap["rec"] = self.rec[seq.slot].clone()
            snap["conv"] = self.conv[seq.slot].clone()
        return snap

    def prefix_snapshot(self, seq: SeqState, pos: int) -> dict:
        """Checkpoint of the first ``pos`` committed tokens: GDN state + conv window (copies) and
        the KV blocks below ``pos`` (shared, reference-counted).  ``pos`` must equal the committed
        length and sit on a KV block boundary."""
        if pos != seq.pos or pos % self.block_size:
            raise ValueError("prefix snapshots are taken at the committed frontier on a block boundary")
        blocks = list(seq.blocks[:pos // self.block_size])
        self.allocator.incref(blocks)
        snap = self.snapshot(seq)
        snap["blocks"] = blocks
        snap["nbytes"] = sum(t.numel() * t.element_size() for k, t in snap.items() if torch.is_tensor(t))
        return snap

    def release_prefix(self, snap: dict):
        self.allocator.release(snap.get("blocks", []))
        snap["blocks"] = []

    def sequence_from_prefix(self, snap: dict) -> SeqState:
        """New sequence whose first ``snap['pos']`` tokens reuse the checkpoint's KV blocks and
        state; later positions get blocks of their own."""
        seq = self.new_sequence()
        blocks = list(snap["blocks"])
        self.allocator.incref(blocks)
        seq.blocks = blocks
        if blocks:
            seq.block_table[:len(blocks)] = torch.tensor(blocks, dtype=torch.int32, device=self.device)
        self.restore(seq, snap)
        return seq

    def restore(self, seq: SeqState, snap: dict):
        if hasattr(self, "rec"):
            self.rec[seq.slot].copy_(snap["rec"])
            self.conv[seq.slot].copy_(snap["conv"])
        seq.pos = snap["pos"]
        seq.verify_rows = None

    # ------------------------------------------------------------------ convenience
    @torch.no_grad()
    def sampling_args(self, temperature: float, seed: int, positions):
        """(scale, key) device tensors for sampled rows at ``positions`` (temperature > 0)."""
        from ..ops.torch_ref import sample_key
        n = len(positions)
        scale = torch.full((n,), 1.0 / temperature if temperature > 0 else 0.0, dtype=torch.float32)
        key = torch.tensor([sample_key(seed, int(p)) for p in positions], dtype=torch.int64)
        return scale.to(self.device, non_blocking=True), key.to(self.device, non_blocking=True)

    @torch.no_grad()
    def sample(self, tokens: torch.Tensor, max_new_tokens: int, temperature: float, seed: int = 0, eos=None):
        """Plain (non-speculative) decoding that samples every token from softmax(logits / T) by
        Gumbel-max inside the LM-head kernel; the token at position p uses the noise key
        (seed, p), so a sample does not depend on batching or tensor parallelism."""
        if temperature <= 0:
            return self.greedy(tokens, max_new_tokens, eos)
        seq = self.new_sequence()
        try:
            n = int(tokens.shape[0])
            nxt, _ = self.prefill(seq, tokens, sampling=self.sampling_args(temperature, seed, [n]))
            out = [int(nxt.item())]
            while len(out) < max_new_tokens and (eos is None or out[-1] != eos):
                p = seq.pos + 1                     # position of the token this step produces
                pred, _ = self.verify([(seq, torch.tensor([out[-1]], device=self.device))],
                                      sampling=self.sampling_args(temperature, seed, [p]))
                self.commit(seq, 1)
                out.append(int(pred[0].item()))
            return out
        finally:
            self.release(seq)

    def greedy(self, tokens: torch.Tensor, max_new_tokens: int, eos=None):
        seq = self.new_sequence()
        try:
            nxt, _ = self.prefill(seq, tokens)
            out = [int(nxt.item())]
            while len(out) < max_new_tokens and (eos is None or out[-1] != eos):
                nxt, _ = self.decode(seq, torch.tensor([out[-1]], device=self.device))
                out.append(int(nxt.item()))
            return out
        finally:
            self.release(seq)
