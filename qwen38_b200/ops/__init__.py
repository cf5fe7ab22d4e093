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
    def linear(self, x, w, out_dtype=None):
        y = x @ w.t()
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

    def lm_head_argmax(self, x, w, vocab_offset: int = 0):
        """Returns (max value fp32 [T], global index int64 [T]); ties take the lowest index."""
        logits = (x @ w.t()).float()
        v, i = logits.max(-1)
        return v, i + vocab_offset

    # ---- norms ---------------------------------------------------------------------
    def rms_norm(self, x, w_eff, eps, out_dtype):
        """y = x * rsqrt(mean(x^2)+eps) * w_eff  (w_eff already holds 1+w where applicable)."""
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w_eff
        return y.to(out_dtype)

    def embedding(self, ids, table):
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
    def attn_prep(self, proj, qn_w, kn_w, cos, sin, dims, eps, kcache, vcache, block_table, pos0, block_size):
        """Split [q | gate | k | v] rows, q/k (1+w) RMSNorm, partial RoPE, write K/V rows into
        the paged cache at positions pos0..pos0+T-1.  Returns q [T, H, D], gate [T, H*D]."""
        H, Hkv, D = dims
        T = proj.shape[0]
        q = proj[:, :H * D].reshape(T, H, D)
        gate = proj[:, H * D:2 * H * D]
        k = proj[:, 2 * H * D:2 * H * D + Hkv * D].reshape(T, Hkv, D)
        v = proj[:, 2 * H * D + Hkv * D:2 * H * D + 2 * Hkv * D].reshape(T, Hkv, D)
        q = self.rms_norm(q, qn_w, eps, torch.float32)   # qn_w / kn_w hold 1+w
        k = self.rms_norm(k, kn_w, eps, torch.float32)
        q = R.apply_rope(q, cos, sin).to(proj.dtype)
        k = R.apply_rope(k, cos, sin).to(kcache.dtype)
        pos = torch.arange(pos0, pos0 + T, device=proj.device)
        blk = block_table[(pos // block_size).long()].long()
        off = pos % block_size
        kcache[blk, off] = k
        vcache[blk, off] = v.to(vcache.dtype)
        return q, gate

    def attn_decode(self, q, gate, kcache, vcache, block_table, pos0, block_size, out_dtype):
        """Row t (position pos0+t) attends cache keys 0..pos0+t; output times sigmoid(gate)."""
        T, H, D = q.shape
        S = pos0 + T
        pos = torch.arange(S, device=q.device)
        blk = block_table[(pos // block_size).long()].long()
        K = kcache[blk, pos % block_size]
        V = vcache[blk, pos % block_size]
        qpos = torch.arange(pos0, pos0 + T, device=q.device)
        o = R.attention(q, K, V, qpos, pos, D ** -0.5, causal=True)
        o = o.reshape(T, H * D) * torch.sigmoid(gate.float())
        return o.to(out_dtype)

    attn_prefill = attn_decode

    def draft_attention(self, q, kctx, vctx, n_ctx, k_blk, v_blk, scale, out_dtype):
        """Every block row attends all ``n_ctx`` history rows plus every block row (no mask)."""
        P, H, D = q.shape
        K = torch.cat([kctx[:n_ctx], k_blk.to(kctx.dtype)], 0)
        V = torch.cat([vctx[:n_ctx], v_blk.to(vctx.dtype)], 0)
        pos = torch.zeros(K.shape[0], device=q.device)
        o = R.attention(q, K, V, torch.zeros(P, device=q.device), pos, scale, causal=False)
        return o.reshape(P, H * D).to(out_dtype)

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
