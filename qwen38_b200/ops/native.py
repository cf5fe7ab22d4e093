"""``NativeOps``: the runtime's op set on the hand-written sm_100a kernels.

Requires CUDA tensors and the in-tree extension (``qwen38_b200/_build``); there is no fallback.
Scratch buffers (split-K partials and counters, attention split partials, argmax partials, the
device error word) are allocated once per device so every launch is graph-capturable.

``launches`` counts the kernels this op set enqueued (bench ``gpu_launches``).
"""
from __future__ import annotations

import torch

from . import TorchOps
from . import torch_ref as R
from .build import load

EPI_BF16, EPI_F32, EPI_ADD_F32, EPI_SWIGLU, EPI_ARGMAX = range(5)


class KernelError(RuntimeError):
    pass


class TiledWeight:
    """A GEMM weight of logical shape [N, K] stored tile-contiguous for the tcgen05 kernels:
    tile (n // 128, k // 64) is one contiguous 16 KB block, so every TMA load of a weight tile is
    a single contiguous stream.  Rows / columns are zero-padded to multiples of 128 / 64."""
    __slots__ = ("t", "N", "K")

    def __init__(self, t, N, K):
        self.t, self.N, self.K = t, N, K

    @property
    def shape(self):
        return (self.N, self.K)


def tile_weight(w: torch.Tensor) -> TiledWeight:
    N, K = w.shape
    NT, KB = -(-N // 128), -(-K // 64)
    if N % 128 or K % 64:
        wp = torch.zeros(NT * 128, KB * 64, dtype=w.dtype, device=w.device)
        wp[:N, :K] = w
    else:
        wp = w
    t = wp.reshape(NT, 128, KB, 64).permute(0, 2, 1, 3).contiguous().view(NT * KB * 128, 64)
    return TiledWeight(t, N, K)


class MXWeight:
    """An MXFP8 GEMM weight of logical shape [N, K] (e4m3 values, one E8M0 scale per 32 elements of
    a row) for the weight-streaming GEMM, stored like a TiledWeight: tile (n // 128, k // 64) is one
    contiguous 8 KB block of e4m3 bytes ``q`` and one 256-byte block of scales ``s`` ([128 rows][2]).
    ``t`` is the exact bf16 expansion in TiledWeight layout, read by the prefill-tile GEMMs (which
    are compute-bound and take bf16 operands); the <= 64-row GEMMs stream ``q`` and ``s``."""
    __slots__ = ("q", "s", "t", "N", "K")

    def __init__(self, q, s, t, N, K):
        self.q, self.s, self.t, self.N, self.K = q, s, t, N, K

    @property
    def shape(self):
        return (self.N, self.K)


def mx_tile_weight(w: torch.Tensor, bf16: TiledWeight | None = None):
    """MXWeight of ``w`` when its values are exactly an MXFP8 tensor with the OCP scale choice
    (so storing it as MXFP8 loses nothing), else None.  Scales above 2^7 are refused (the kernel's
    bf16 rescale factor 2^(scale + 120) must stay a normal bf16)."""
    from ..checkpoint import dequant_mxfp8, quant_mxfp8
    N, K = w.shape
    wf = w.float()
    q, se = quant_mxfp8(wf)
    if int(se.max()) > 134 or not torch.equal(dequant_mxfp8(q, se), wf):
        return None
    NT, KB = -(-N // 128), -(-K // 64)
    qb = torch.zeros(NT * 128, KB * 64, dtype=torch.uint8, device=w.device)
    qb[:N, :K] = q.view(torch.uint8)
    sb = torch.zeros(NT * 128, KB * 2, dtype=torch.uint8, device=w.device)
    sb[:N, :se.shape[1]] = se
    qt = qb.reshape(NT, 128, KB, 64).permute(0, 2, 1, 3).contiguous().view(NT * KB * 128, 64)
    st = sb.reshape(NT, 128, KB, 2).permute(0, 2, 1, 3).contiguous().view(NT * KB * 128, 2)
    t = (bf16 or tile_weight(w.to(torch.bfloat16).contiguous())).t
    return MXWeight(qt, st, t, N, K)


def untile_weight(tw: TiledWeight) -> torch.Tensor:
    NT, KB = -(-tw.N // 128), -(-tw.K // 64)
    return tw.t.view(NT, KB, 128, 64).permute(0, 2, 1, 3).reshape(NT * 128, KB * 64)[:tw.N, :tw.K]


_ERR_NAMES = {1: "TMA/mbarrier wait timeout", 2: "accumulator wait timeout", 4: "split-K fix-up timeout",
              8: "peer flag timeout", 16: "unsupported shape or out-of-range cache position"}


class NativeOps(TorchOps):
    name = "native"
    # token rows the weight-streaming (swap-AB) GEMM, the cluster norms and the pushed all-reduce
    # serve (csrc SWAP_MAX_ROWS / AR_MAX_ROWS): a packed verify of up to 4 x 16 rows stays on them
    max_pack_rows = 64

    def __init__(self, device=None, max_keys: int = 1 << 17, ws_mb: int = 64, weight_format: str = "bf16"):
        if weight_format not in ("bf16", "mxfp8"):
            raise ValueError("weight_format must be bf16 or mxfp8")
        # mxfp8: every GEMM weight whose values are exactly MXFP8 is kept as MXFP8 and streamed at
        # one byte per element by the <= 64-row GEMMs
        self.weight_format = weight_format
        self.C = load()
        if not torch.cuda.is_available():
            raise RuntimeError("NativeOps needs a CUDA device")
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        dev = self.device
        self.ws = torch.zeros(ws_mb << 18, dtype=torch.float32, device=dev)          # ws_mb MiB
        self.counters = torch.zeros(1 << 16, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.amax_val = torch.empty(1 << 20, dtype=torch.float32, device=dev)
        self.amax_idx = torch.empty(1 << 20, dtype=torch.int32, device=dev)
        self.max_keys = max_keys
        self._attn_bufs = {}
        self.rows_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self.markov_state = torch.zeros(4 + 32, dtype=torch.int32, device=dev)   # grid barrier + epochs
        self.launches = 0
        self.chunked_prefill = True
        self._gdn_work = None
        self._split_parts = None          # deferred split-K slices [8][64][N] fp32 (linear_split)

    # ------------------------------------------------------------------ errors
    def check(self):
        e = int(self.err.item())
        if e:
            names = [n for b, n in _ERR_NAMES.items() if e & b]
            self.err.zero_()
            self.counters.zero_()
            self.markov_state[:2].zero_()          # a grid barrier that gave up may be mid-count
            raise KernelError(f"device error word {e}: {', '.join(names)}")

    # ------------------------------------------------------------------ GEMMs
    def prepare_weight(self, w):
        if isinstance(w, (TiledWeight, MXWeight)):
            return w
        if self.weight_format == "mxfp8" and w.dim() == 2:
            mw = mx_tile_weight(w)
            if mw is not None:
                return mw
        return tile_weight(w.to(torch.bfloat16).contiguous())

    @staticmethod
    def _mx(w, T):
        """True when this GEMM streams the MX bytes of ``w`` (an MXWeight, <= 64 rows)."""
        return isinstance(w, MXWeight) and T <= NativeOps.max_pack_rows

    def linear(self, x, w, out_dtype=None, out=None):
        w = self.prepare_weight(w)
        x = x.contiguous()
        T, N = x.shape[0], w.N
        if out_dtype == torch.float32 or (out is not None and out.dtype == torch.float32):
            if out is None:
                out = torch.empty(T, N, dtype=torch.float32, device=x.device)
            epi = EPI_F32
        else:
            if out is None:
                out = torch.empty(T, N, dtype=torch.bfloat16, device=x.device)
            epi = EPI_BF16
        if self._mx(w, T):
            self.C.linear_mx(x, w.q, w.s, N, out, epi, self.ws, self.counters, self.err)
        else:
            self.C.linear(x, w.t, N, out, epi, self.ws, self.counters, self.err)
        self.launches += 1
        return out

    def linear_push(self, x, w, comm) -> int:
        """GEMM half of the tensor-parallel all-reduce: x @ w^T (fp32, T <= 64 rows) goes straight
        from each finished tile into every rank's receive block of a fresh slot as {value, epoch}
        words; returns the slot for ``rms_norm_ar``."""
        w = self.prepare_weight(w)
        slot = comm.fused_slot()
        mx = self._mx(w, x.shape[0])
        self.C.linear_push(x.contiguous(), w.q if mx else w.t, w.N, self.ws, self.counters, self.err, comm.recv_ptrs,
                           comm.rank, slot, comm.block_words, comm.fepochs, int(getattr(comm, "recv_mc", 0) or 0),
                           w.s if mx else None)
        self.launches += 1
        return slot

    def rms_norm_ar(self, x, w, eps, out_dtype, comm, slot):
        """Reduction half: waits for every rank's words of ``slot``, adds them (rank order) into the
        fp32 residual ``x`` in place and returns RMSNorm(x) * w in bf16 (``w`` None: reduce only)."""
        out = None if w is None else torch.empty(x.shape[0], x.shape[1], dtype=torch.bfloat16, device=x.device)
        self.C.rms_norm_ar(x, w, float(eps), out, comm.recv_ptrs[comm.rank], comm.fepochs, slot, comm.world,
                           comm.block_words, self.err)
        self.launches += 1
        return out if out is None or out_dtype == torch.bfloat16 else out.to(out_dtype)

    def linear_residual(self, x, w, residual):
        w = self.prepare_weight(w)
        if self._mx(w, x.shape[0]):
            self.C.linear_mx(x.contiguous(), w.q, w.s, w.N, residual, EPI_ADD_F32, self.ws, self.counters, self.err)
        else:
            self.C.linear(x.contiguous(), w.t, w.N, residual, EPI_ADD_F32, self.ws, self.counters, self.err)
        self.launches += 1
        return residual

    def linear_split(self, x, w, residual) -> int:
        """residual += x @ w^T for <= 64 rows with the split-K reduction deferred: each K slice of
        the GEMM stores its fp32 partial and exits; ``rms_norm_split`` adds the slices (split order)
        and the residual, the bits of ``linear_residual``.  Returns the slice count S; with S == 1
        the GEMM has added into ``residual`` already and nothing is pending."""
        w = self.prepare_weight(w)
        T, N = residual.shape
        need = 8 * self.max_pack_rows * N
        if self._split_parts is None or self._split_parts.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("linear_split: slice buffer must be sized before graph capture")
            self._split_parts = torch.empty(need, dtype=torch.float32, device=self.device)
        mx = self._mx(w, T)
        S = int(self.C.linear_split(x.contiguous(), w.q if mx else w.t, w.N, residual, self._split_parts, self.ws,
                                    self.counters, self.err, w.s if mx else None))
        self.launches += 1
        return S

    def rms_norm_split(self, x, w, eps, out_dtype, S):
        """Completes a pending ``linear_split`` of S slices into the residual ``x`` and returns
        RMSNorm(x) * w in bf16 (``w`` None: completes the residual only)."""
        out = None if w is None else torch.empty(x.shape[0], x.shape[1], dtype=torch.bfloat16, device=x.device)
        self.C.rms_norm_split(x, self._split_parts, int(S), w, float(eps), out)
        self.launches += 1
        return out if out is None or out_dtype == torch.bfloat16 else out.to(out_dtype)

    def linear_swiglu(self, x, w_gu, block):
        if block != 64:
            raise ValueError("the SwiGLU epilogue pairs 64-row gate/up blocks")
        w_gu = self.prepare_weight(w_gu)
        x = x.contiguous()
        out = torch.empty(x.shape[0], w_gu.N // 2, dtype=torch.bfloat16, device=x.device)
        if self._mx(w_gu, x.shape[0]):
            self.C.linear_mx(x, w_gu.q, w_gu.s, w_gu.N, out, EPI_SWIGLU, self.ws, self.counters, self.err)
        else:
            self.C.linear(x, w_gu.t, w_gu.N, out, EPI_SWIGLU, self.ws, self.counters, self.err)
        self.launches += 1
        return out

    def lm_head_argmax(self, x, w, vocab_offset=0, sampling=None):
        """Per row (max value, global index) of x @ w^T; rows with a positive scale in ``sampling``
        = (scale [T] fp32, key [T] int64) take Gumbel-max samples of softmax(logits * scale)."""
        w = self.prepare_weight(w)
        x = x.contiguous()
        T = x.shape[0]
        val = torch.empty(T, dtype=torch.float32, device=x.device)
        idx = torch.empty(T, dtype=torch.int64, device=x.device)
        sc, key = sampling if sampling is not None else (None, None)
        self.C.lm_head_argmax(x, w.t, w.N, val, idx, int(vocab_offset), self.amax_val, self.amax_idx, self.ws,
                              self.counters, self.err, sc, key)
        self.launches += 2
        return val, idx

    # ------------------------------------------------------------------ norms / embedding
    def rms_norm(self, x, w_eff, eps, out_dtype):
        if out_dtype != torch.bfloat16:
            return super().rms_norm(x, w_eff, eps, out_dtype)
        x2 = x.reshape(-1, x.shape[-1])
        out = torch.empty(x2.shape, dtype=torch.bfloat16, device=x.device)
        self.C.rms_norm(x2, w_eff, float(eps), out)
        self.launches += 1
        return out.reshape(x.shape)

    def embedding(self, ids, table, out=None):
        if out is None:
            out = torch.empty(ids.numel(), table.shape[1], dtype=torch.float32, device=ids.device)
        self.C.embedding(ids.reshape(-1).long(), table, out)
        self.launches += 1
        return out

    # ------------------------------------------------------------------ GDN
    def gdn_verify(self, proj, window, state, conv_w, A_log, dt_bias, norm_w, eps, dims, out_dtype):
        nk, nv, dk, dv = dims
        out = torch.empty(proj.shape[0], nv * dv, dtype=torch.bfloat16, device=proj.device)
        self.C.gdn_recurrent(0, proj, window, state, conv_w, A_log, dt_bias, norm_w, out, proj.shape[0], None,
                             nk, nv, dk, float(eps))
        self.launches += 1
        return out

    def gdn_prefill(self, proj, window, state, conv_w, A_log, dt_bias, norm_w, eps, dims, chunk, out_dtype):
        """Committed prefill: the chunked tensor-core kernels for head dim 128, the sequential
        recurrence otherwise (small test shapes)."""
        nk, nv, dk, dv = dims
        S = proj.shape[0]
        out = torch.empty(S, nv * dv, dtype=torch.bfloat16, device=proj.device)
        if dk == 128 and dv == 128 and self.chunked_prefill:
            need = int(self.C.gdn_chunk_workspace_bytes(S, nv))
            if self._gdn_work is None or self._gdn_work.numel() < need:
                self._gdn_work = torch.empty(need, dtype=torch.uint8, device=proj.device)
            C = conv_w.shape[0]
            self.C.gdn_chunk_prefill(proj, window, state, conv_w, A_log, dt_bias, norm_w, out, self._gdn_work,
                                     nk, nv, float(eps))
            K1 = window.shape[0]
            if S >= K1:
                window.copy_(proj[S - K1:, :C])
            else:
                window.copy_(torch.cat([window[S:], proj[:, :C]], 0))
            self.launches += 4
            return out
        self.C.gdn_recurrent(2, proj, window, state, conv_w, A_log, dt_bias, norm_w, out, S, None,
                             nk, nv, dk, float(eps))
        self.launches += 2
        return out

    def gdn_commit(self, proj, n, window, state, conv_w, A_log, dt_bias, dims):
        nk, nv, dk, dv = dims
        self.rows_dev.fill_(int(n))
        dummy_norm = torch.empty(dv, dtype=torch.float32, device=proj.device)
        self.C.gdn_recurrent(1, proj, window, state, conv_w, A_log, dt_bias, dummy_norm, None, int(n),
                             self.rows_dev, nk, nv, dk, 1e-6)
        self.launches += 2

    def gdn_commit_layers(self, stash, n, conv, rec, conv_w, A_log, dt_bias, dims):
        nk, nv, dk, dv = dims
        self.rows_dev.fill_(int(n))
        norm_dummy = torch.empty(rec.shape[0], dv, dtype=torch.float32, device=rec.device)
        self.C.gdn_recurrent(1, stash, conv, rec, conv_w, A_log, dt_bias, norm_dummy, None, int(n), self.rows_dev,
                             nk, nv, dk, 1e-6)
        self.launches += 2

    # ------------------------------------------------------------------ attention
    def _bufs(self, nkv, nqv, D):
        key = (nkv, nqv, D)
        b = self._attn_bufs.get(key)
        if b is None:
            splits = -(-self.max_keys // 128)   # 128-key chunks (csrc/attention.cu CH)
            b = (torch.empty(nkv * splits * nqv * D, dtype=torch.float32, device=self.device),
                 torch.empty(nkv * splits * nqv * 2, dtype=torch.float32, device=self.device))
            self._attn_bufs[key] = b
        return b

    def attn_prep(self, proj, qn_w, kn_w, inv_freq, rope_scale, rd, dims, eps, positions, kcache, vcache,
                  block_table, block_size):
        H, Hkv, D = dims
        T = proj.shape[0]
        q = torch.empty(T, H, D, dtype=torch.bfloat16, device=proj.device)
        self.C.attn_prep(proj, 0, 2 * H * D, 2 * H * D + Hkv * D, H, Hkv, D, rd, qn_w, kn_w, inv_freq,
                         float(rope_scale), float(eps), positions, q, kcache, vcache, block_table, block_size,
                         self.err)
        self.launches += 1
        return q, proj[:, H * D:2 * H * D]

    def attn_decode(self, q, gate, kcache, vcache, block_table, positions, block_size, out_dtype, causal=True):
        T, H, D = q.shape
        if T > 32:
            return self.attn_prefill(q, gate, kcache, vcache, block_table, positions, block_size, out_dtype)
        nkv = kcache.shape[-2]
        po, pml = self._bufs(nkv, H // nkv * T, D)
        out = torch.empty(T, H * D, dtype=torch.bfloat16, device=q.device)
        g = gate
        self.C.attn_decode(q, kcache, vcache, block_table, block_size, positions, D ** -0.5, int(causal), g,
                           0, out, po, pml, self.max_keys, self.err)
        self.launches += 2
        return out

    def attn_prefill(self, q, gate, kcache, vcache, block_table, positions, block_size, out_dtype):
        """Causal prefill attention of a chunk over the paged cache (``attn_prefill_kernel``:
        flash attention on tensor cores, GQA heads of a KV head in one CTA, sigmoid-gate epilogue)."""
        T, H, D = q.shape
        out = torch.empty(T, H * D, dtype=torch.bfloat16, device=q.device)
        self.C.attn_prefill(q.contiguous(), kcache, vcache, block_table, block_size, positions, D ** -0.5, gate, out)
        self.launches += 1
        return out if out_dtype == torch.bfloat16 else out.to(out_dtype)

    def kv_append(self, kv, kn_w, inv_freq, rope_scale, rd, nkv, D, eps, positions, kcache, vcache):
        self.C.attn_prep(kv, -1, 0, nkv * D, 0, nkv, D, rd, kn_w, kn_w, inv_freq, float(rope_scale), float(eps),
                         positions, None, kcache, vcache, None, 0, self.err)
        self.launches += 1

    def draft_block_attention(self, qkv, qn_w, kn_w, inv_freq, rope_scale, dims, eps, positions, kcache, vcache,
                              out_dtype, window: int = 0):
        H, Hkv, D = dims
        T = qkv.shape[0]
        q = torch.empty(T, H, D, dtype=torch.bfloat16, device=qkv.device)
        self.C.attn_prep(qkv, 0, H * D, (H + Hkv) * D, H, Hkv, D, D, qn_w, kn_w, inv_freq, float(rope_scale),
                         float(eps), positions, q, kcache, vcache, None, 0, self.err)
        po, pml = self._bufs(Hkv, H // Hkv * T, D)
        out = torch.empty(T, H * D, dtype=torch.bfloat16, device=qkv.device)
        if window > 0:
            self.C.attn_decode_window(q, kcache, vcache, None, 0, positions, D ** -0.5, 0, None, 0, out, po, pml,
                                      self.max_keys, int(window), self.err)
        else:
            self.C.attn_decode(q, kcache, vcache, None, 0, positions, D ** -0.5, 0, None, 0, out, po, pml,
                               self.max_keys, self.err)
        self.launches += 3
        return out

    def draft_conv(self, x, dyn, tap0: int, base, group: int, residual=None, out_dtype=torch.bfloat16):
        if residual is None:
            if out_dtype != torch.bfloat16:
                raise ValueError("the native convolution writes bf16 rows")
            out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
            self.C.draft_conv(x.contiguous(), dyn, int(tap0), base, int(group), out, None)
        else:
            out = residual
            self.C.draft_conv(x.contiguous(), dyn, int(tap0), base, int(group), None, residual)
        self.launches += 1
        return out

    def draft_select(self, feats, cand, unary, anchor, pred, succ):
        out = torch.empty(cand.shape[0] - 1, dtype=torch.int64, device=cand.device)
        self.C.draft_select(feats, cand.contiguous(), unary.contiguous(), anchor.reshape(-1), pred, succ, out,
                            self.err)
        self.launches += 1
        return out

    # ------------------------------------------------------------------ sampling
    def markov_select(self, logits, anchor, pred, succ, vocab_offset=0, comm=None):
        """All P sequential Markov steps in one persistent launch (``csrc/markov.cu``); at TP > 1
        each step's cross-rank argmax runs inside the launch over the peer-memory words of
        ``comm.markov_ptrs``.  A communicator without peer memory takes the per-step kernels and
        the communicator's argmax."""
        P = logits.shape[0]
        if comm is None or hasattr(comm, "markov_ptrs"):
            out = torch.empty(P, dtype=torch.int64, device=logits.device)
            a = anchor.reshape(1)
            if a.dtype != torch.int64:
                a = a.long()
            self.C.markov_select(logits if logits.stride(1) == 1 else logits.contiguous(), pred, succ, a, out,
                                 int(vocab_offset), self.amax_val, self.amax_idx, self.markov_state,
                                 list(comm.markov_ptrs) if comm is not None else [],
                                 int(comm.rank) if comm is not None else 0, self.err)
            self.launches += 1
            return out
        prev = anchor.reshape(1).clone().long()
        out = torch.empty(P, dtype=torch.int64, device=logits.device)
        val = torch.empty(1, dtype=torch.float32, device=logits.device)
        for i in range(P):
            self.C.markov_step(logits[i].contiguous(), pred, succ, prev, out[i:i + 1], val, self.amax_val,
                               self.amax_idx, int(vocab_offset), comm is None)
            self.launches += 2
            if comm is not None:
                g = comm.argmax_reduce(val, out[i:i + 1])
                out[i:i + 1].copy_(g)
                prev.copy_(g)
        return out
