"""Op sets used by the runtime.

``TorchOps`` states every fused op with plain PyTorch (cuBLAS for GEMMs on a GPU): it runs the
CPU/gloo paths and is the "NCCL + cuBLAS" baseline build on a B200.  ``NativeOps``
(``qwen38_b200.ops.native``) runs the hand-written sm_100a kernels and refuses to run without
its compiled extension.  The runtime picks one explicitly; nothing falls back silently.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import torch_ref as R


class TorchOps:
    name = "torch"

    # ---- GEMM family: y = x @ w^T ------------------------------------------------
    def prepare_weight(self, w):
        """Storage layout of a GEMM weight for this op set (identity here)."""
        return w

    def linear(self, x, w, out_dtype=None, out=None):
        y = x @ w.t()
        if out is not None:
            out.copy_(y)
            return out
        return y if out_dtype is None else y.to(out_dtype)

    def linear_residual(self, x, w, residual):
        """residual += x @ w^T (fp32 residual)."""
        residual += (x.float() @ w.float().t()) if x.device.type == "cpu" else (x @ w.t()).float()
        return residual

    def linear_swiglu(self, x, w_gu, block: int):
        """w_gu rows are [gate 'block' | up 'block'] per feature block; returns silu(g)*u."""
        y = x @ w_gu.t()
        T = y.shape[0]
        y = y.view(T, -1, 2, block)
        return R.swiglu(y[:, :, 0], y[:, :, 1]).reshape(T, -1)

    def lm_head_argmax(self, x, w, vocab_offset: int = 0, sampling=None):
        """Returns (max value fp32 [T], global index int64 [T]); ties take the lowest index.
        ``sampling`` = (scale [T], key [T]): rows with scale > 0 take argmax(logits * scale +
        Gumbel noise(key, global index)), a sample of softmax(logits * scale)."""
        logits = (x @ w.t()).float()
        if sampling is not None:
            sc, key = sampling
            sc = sc.to(logits.device).float()
            rows = sc > 0
            if bool(rows.any()):
                idx = torch.arange(vocab_offset, vocab_offset + logits.shape[1], device=logits.device)
                g = R.gumbel_noise(key.to(logits.device), idx)
                logits = torch.where(rows[:, None], logits * sc[:, None] + g, logits)
        v, i = logits.max(-1)
        return v, i + vocab_offset

    # ---- norms ---------------------------------------------------------------------
    def rms_norm(self, x, w_eff, eps, out_dtype):
        """y = x * rsqrt(mean(x^2)+eps) * w_eff  (w_eff already holds 1+w where applicable)."""
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w_eff
        return y.to(out_dtype)

    def embedding(self, ids, table, out=None):
        if out is not None:
            out.copy_(table[ids])
            return out
        return table[ids]

    # ---- GDN -----------------------------------------------------------------------
    def gdn_prepare(self, proj, window, conv_w, A_log, dt_bias, dims):
        """From in-projection rows [T, C_in] (layout q|k|v|z|b|a) and the conv window [K-1, C]:
        returns q, k (L2-normalised, q scaled, expanded to value heads) [T, Nv, Dk] fp32,
        v [T, Nv, Dv] fp32, z [T, Nv, Dv], g, beta [T, Nv] fp32, new window."""
        nk, nv, dk, dv = dims
        T = proj.shape[0]
        C = 2 * nk * dk + nv * dv
        qkv = proj[:, :C]
        z = proj[:, C:C + nv * dv].reshape(T, nv, dv)
        b = proj[:, C + nv * dv:C + nv * dv + nv]
        a = proj[:, C + nv * dv + nv:C + nv * dv + 2 * nv]
        y, new_window = R.causal_conv1d(qkv, conv_w, window)
        q = y[:, :nk * dk].reshape(T, nk, dk)
        k = y[:, nk * dk:2 * nk * dk].reshape(T, nk, dk)
        v = y[:, 2 * nk * dk:].reshape(T, nv, dv)
        rep = nv // nk
        q = R.l2norm(q).repeat_interleave(rep, 1) * (dk ** -0.5)
        k = R.l2norm(k).repeat_interleave(rep, 1)
        g, beta = R.gdn_gates(a, b, A_log, dt_bias)
        return q, k, v, z, g, beta, new_window

    def gdn_verify(self, proj, window, state, conv_w, A_log, dt_bias, norm_w, eps, dims, out_dtype):
        """Uncommitted T-row step: outputs gated-normed rows [T, Nv*Dv]; state/window untouched."""
        nk, nv, dk, dv = dims
        q, k, v, z, g, beta, _ = self.gdn_prepare(proj, window, conv_w, A_log, dt_bias, dims)
        o, _ = R.gdn_recurrent(q, k, v, g, beta, state)
        return R.gated_rms_norm(o, z, norm_w, eps).to(out_dtype).reshape(proj.shape[0], nv * dv)

    def gdn_commit(self, proj, n, window, state, conv_w, A_log, dt_bias, dims):
        """Advance state and window in place by the first n rows of ``proj``."""
        if n <= 0:
            return
        q, k, v, z, g, beta, new_window = self.gdn_prepare(proj[:n], window, conv_w, A_log, dt_bias, dims)
        _, S = R.gdn_recurrent(q, k, v, g, beta, state)
        state.copy_(S)
        window.copy_(new_window)

    def gdn_prefill(self, proj, window, state, conv_w, A_log, dt_bias, norm_w, eps, dims, chunk, out_dtype):
        """Committed chunked prefill: returns outputs, advances state/window in place."""
        nk, nv, dk, dv = dims
        q, k, v, z, g, beta, new_window = self.gdn_prepare(proj, window, conv_w, A_log, dt_bias, dims)
        o, S = R.gdn_chunked(q, k, v, g, beta, state, chunk)
        state.copy_(S)
        window.copy_(new_window)
        return R.gated_rms_norm(o, z, norm_w, eps).to(out_dtype).reshape(proj.shape[0], nv * dv)

    # ---- attention -------------------------------------------------------------------
    def attn_prep(self, proj, qn_w, kn_w, inv_freq, rope_scale, rd, dims, eps, positions, kcache, vcache,
                  block_table, block_size):
        """Split [q | gate | k | v] rows, q/k RMSNorm (multiplier weights), partial RoPE at
        ``positions`` [T] (int32), write K/V rows into the cache (paged via ``block_table``, or
        contiguous when it is None).  Returns q [T, H, D] and the gate columns [T, H*D]."""
        H, Hkv, D = dims
        T = proj.shape[0]
        q = proj[:, :H * D].reshape(T, H, D)
        gate = proj[:, H * D:2 * H * D]
        k = proj[:, 2 * H * D:2 * H * D + Hkv * D].reshape(T, Hkv, D)
        v = proj[:, 2 * H * D + Hkv * D:2 * H * D + 2 * Hkv * D].reshape(T, Hkv, D)
        cos, sin = R.rope_cos_sin(positions, rd, 1.0, inv_freq, rope_scale)
        q = R.apply_rope(self.rms_norm(q, qn_w, eps, torch.float32), cos, sin).to(proj.dtype)
        k = R.apply_rope(self.rms_norm(k, kn_w, eps, torch.float32), cos, sin).to(kcache.dtype)
        self._write_kv(k, v, positions, kcache, vcache, block_table, block_size)
        return q, gate

    def _write_kv(self, k, v, positions, kcache, vcache, block_table, block_size):
        pos = positions.long()
        if block_table is None:
            kcache[pos] = k.to(kcache.dtype)
            vcache[pos] = v.to(vcache.dtype)
        else:
            blk = block_table[pos // block_size].long()
            kcache[blk, pos % block_size] = k.to(kcache.dtype)
            vcache[blk, pos % block_size] = v.to(vcache.dtype)

    def _gather_kv(self, kcache, vcache, block_table, block_size, n):
        pos = torch.arange(n, device=kcache.device)
        if block_table is None:
            return kcache[:n], vcache[:n]
        blk = block_table[pos // block_size].long()
        return kcache[blk, pos % block_size], vcache[blk, pos % block_size]

    def attn_decode(self, q, gate, kcache, vcache, block_table, positions, block_size, out_dtype, causal=True):
        """Row t attends cache keys 0..positions[t] (causal) or 0..positions[-1] (full);
        output times sigmoid(gate) when a gate is given."""
        T, H, D = q.shape
        n = int(positions[-1]) + 1
        K, V = self._gather_kv(kcache, vcache, block_table, block_size, n)
        kpos = torch.arange(n, device=q.device)
        o = R.attention(q, K, V, positions.long(), kpos, D ** -0.5, causal=causal)
        o = o.reshape(T, H * D)
        if gate is not None:
            o = o * torch.sigmoid(gate.float())
        return o.to(out_dtype)

    attn_prefill = attn_decode

    def kv_append(self, kv, kn_w, inv_freq, rope_scale, rd, nkv, D, eps, positions, kcache, vcache):
        """Drafter context rows: k = RoPE(RMSNorm(k)), v as is, written contiguously."""
        T = kv.shape[0]
        k = kv[:, :nkv * D].reshape(T, nkv, D)
        v = kv[:, nkv * D:2 * nkv * D].reshape(T, nkv, D)
        cos, sin = R.rope_cos_sin(positions, rd, 1.0, inv_freq, rope_scale)
        k = R.apply_rope(self.rms_norm(k, kn_w, eps, torch.float32), cos, sin)
        self._write_kv(k, v, positions, kcache, vcache, None, 0)

    def draft_block_attention(self, qkv, qn_w, kn_w, inv_freq, rope_scale, dims, eps, positions, kcache, vcache,
                              out_dtype, window: int = 0):
        """Drafter block rows [q | k | v]: norm + RoPE, block K/V written after the history at
        ``positions``, then every block row attends the whole history and every block row (with
        ``window`` > 0: only keys k with position - k < window)."""
        H, Hkv, D = dims
        T = qkv.shape[0]
        q = qkv[:, :H * D].reshape(T, H, D)
        k = qkv[:, H * D:(H + Hkv) * D].reshape(T, Hkv, D)
        v = qkv[:, (H + Hkv) * D:(H + 2 * Hkv) * D].reshape(T, Hkv, D)
        cos, sin = R.rope_cos_sin(positions, D, 1.0, inv_freq, rope_scale)
        q = R.apply_rope(self.rms_norm(q, qn_w, eps, torch.float32), cos, sin).to(qkv.dtype)
        k = R.apply_rope(self.rms_norm(k, kn_w, eps, torch.float32), cos, sin)
        self._write_kv(k, v, positions, kcache, vcache, None, 0)
        if window <= 0:
            return self.attn_decode(q, None, kcache, vcache, None, positions, 0, out_dtype, causal=False)
        n = int(positions[-1]) + 1
        kpos = torch.arange(n, device=q.device)
        o = R.attention(q, kcache[:n], vcache[:n], positions.long(), kpos, D ** -0.5, causal=False, window=window)
        return o.reshape(T, H * D).to(out_dtype)

    def draft_conv(self, x, dyn, tap0: int, base, group: int, residual=None, out_dtype=torch.bfloat16):
        """Windowed drafter's dynamic grouped causal convolution (``torch_ref.draft_conv``) of
        x [R, H] with dynamic kernels dyn [R, >= (tap0 + 2) * H / group] and base [2, H] (fp32):
        an ``out_dtype`` result, or added into the fp32 ``residual``."""
        y = R.draft_conv(x, dyn, tap0, base, group)
        if residual is None:
            return y.to(out_dtype)
        residual += y
        return residual

    def draft_select(self, feats, cand, unary, anchor, pred, succ):
        """Greedy selector over block rows 1..R-1 (fp64, device tensors only, no host sync):
        candidates cand [R, C] (global ids) with logits unary [R, C], selector features feats [R, rank],
        codebooks pred / succ [V, rank]; returns proposal ids [R-1] (int64)."""
        prev = anchor.reshape(1).long()
        out = []
        for i in range(1, cand.shape[0]):
            pv = pred.index_select(0, prev)[0].double() * feats[i].double()
            sv = succ.index_select(0, cand[i]).double()
            sc = unary[i].double() + sv @ pv
            prev = cand[i].index_select(0, torch.argmax(sc).reshape(1))
            out.append(prev)
        return torch.cat(out)

    def gdn_commit_layers(self, stash, n, conv, rec, conv_w, A_log, dt_bias, dims):
        """Commit the first ``n`` rows of every layer's kept projection rows (stacked [L, ...])."""
        for j in range(stash.shape[0]):
            self.gdn_commit(stash[j], n, conv[j], rec[j], conv_w[j], A_log[j], dt_bias[j], dims)

    def check(self):
        pass

    # ---- sampling --------------------------------------------------------------------
    def markov_select(self, logits, anchor, pred, succ, vocab_offset=0, comm=None):
        """Sequential Markov selection over (possibly vocab-sharded) logits [P, V_l]."""
        prev = anchor.reshape(1).long()
        out = []
        for i in range(logits.shape[0]):
            scores = logits[i].float() + succ.float() @ pred[prev[0]].float()
            v, idx = scores.max(-1)
            idx = idx.reshape(1) + vocab_offset
            if comm is not None:
                idx = comm.argmax_reduce(v.reshape(1), idx)
            prev = idx.reshape(1).long()
            out.append(prev)
        return torch.cat(out)


def get_ops(name: str):
    if name == "torch":
        return TorchOps()
    if name == "native":
        from .native import NativeOps
        return NativeOps()
    raise ValueError(f"unknown op set {name!r}")
