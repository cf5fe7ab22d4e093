"""Windowed block drafter (DFlash2 family): a sliding history window, dynamic grouped causal
convolutions around every layer branch, and a learned candidate selector.

The reference ran this drafter before its DSpark drafter replaced it.  Behaviour pinned by its
device drafter (``scripts/ci/dflash_device.py:515-1237``, proposal at ``:1110``), the layer
branches (``scripts/ci/draft_attention_branch.py:47-297``, ``scripts/ci/draft_mlp_branch.py:22-106``),
the convolution oracle (``scripts/ci/draft_convolution.py:17-37``), the window mask
(``scripts/ci/draft_attention.py:4-18``), the candidate head (``scripts/ci/draft_shared_head.py``)
and the selector oracle (``scripts/ci/draft_selector.py``):

1. History: every committed target row is projected once, ``hidden_norm(fc(taps))``, and each
   layer keeps its K/V (k_norm + rotary at the row's absolute position).  Block row i (position
   pos + i) sees history keys k with pos + i - k < window, and every block row.
2. Block rows ``[anchor, MASK, ..., MASK]`` (``block_rows`` of them) at positions pos .. pos+R-1.
   Each layer has an attention and an MLP branch, both framed by the convolution
   ``conv_t(y)[r, c] = (base[t,0,c] + k[r,2t,c//16]) y[r,c] + (base[t,1,c] + k[r,2t+1,c//16]) y[r-1,c]``
   whose dynamic weights ``k = bf16(RMSNorm(x) @ W_kernel^T)`` the branch's own rows produce:
     attention: x += conv_1(o_proj(attention(q, k, v of conv_0(RMSNorm(x)))))
     MLP:       x += conv_1(down(swiglu(gate, up of conv_0(RMSNorm(x)))))
   Block K/V come from the convolved rows; history K/V from the unconvolved history rows.
3. Final norm, then the target's (shared) LM head gives each row's top candidates (global over the
   vocabulary shards, ties to the lower id) and ``bf16(rows @ W_sel^T)`` the selector features.
4. The selector walks rows 1..R-1: candidate c of row i scores
   ``logit(c) + sum_k pred[prev, k] f[i, k] succ[c, k]``, the best becomes the proposal and the
   next ``prev`` (starting from the anchor): R - 1 proposals, one verify block of R rows.

B200 layout: the residual stream stays fp32 between branches (the reference rounds it to bf16
after each branch); the convolutions, the window mask and the selector chain are device kernels
(``csrc/draft_window.cu``, ``attn_decode_kernel<D, true>``), so a whole proposal is one CUDA
graph with no host round trip; history K/V live in the same per-slot buffers as the DSpark
drafter's, so prefix checkpoints and slot handling are shared.  Tensor parallel like the DSpark
drafter: heads split, row-parallel ``o_proj`` / ``down`` summed before the closing convolution,
vocabulary-sharded head with the candidates gathered across ranks; convolution kernels, selector
projection and codebooks replicated.
"""
from __future__ import annotations

import torch

from ..config import WindowDrafterConfig
from .drafter import BlockDrafter, _heads_split
from .target import GU_BLOCK, HybridTarget


class WindowDrafter(BlockDrafter):
    def __init__(self, dcfg: WindowDrafterConfig, src, target: HybridTarget, *, max_context: int | None = None,
                 slots: int = 1):
        self.dcfg, self.target = dcfg, target
        self.ops, self.comm = target.ops, target.comm
        self.device, self.dtype = target.device, target.dtype
        tp, r = target.tp, target.rank
        self.tp = tp
        H, Dh = dcfg.hidden_size, dcfg.head_dim
        if H != target.cfg.hidden_size:
            raise ValueError("drafter width must equal the target hidden size (shared embedding/head)")
        if dcfg.num_attention_heads % tp or dcfg.intermediate_size % (tp * GU_BLOCK):
            raise ValueError("drafter heads / intermediate do not divide by TP")
        if dcfg.candidates > target.widths["vocab"]:
            raise ValueError("more selector candidates than vocabulary entries per rank")
        self.eps = dcfg.rms_norm_eps
        self.P = dcfg.proposals
        self.window, self.group, self.n_cand = dcfg.window, dcfg.conv_group, dcfg.candidates
        self.mask_id = dcfg.mask_id(target.cfg.vocab_size)
        dev, dt = self.device, self.dtype
        f32 = lambda n: src.get(n, device=dev, dtype=torch.float32).float().contiguous()
        get = lambda n: src.get(n, device=dev, dtype=dt)
        pw = self.ops.prepare_weight
        kin = len(dcfg.taps) * H
        if kin % tp:
            raise ValueError("fc input width must divide by TP")
        kl = kin // tp
        fc = get("fc.weight")
        self.fc = pw(fc[:, r * kl:(r + 1) * kl].contiguous())
        del fc
        self.fc_k = (r * kl, kl)
        self.hidden_norm = f32("hidden_norm.weight")
        self.norm = f32("norm.weight")
        hl, kvl, kv_heads = _heads_split(dcfg.num_attention_heads, dcfg.num_key_value_heads, tp, r)
        self.heads = (hl, kvl, Dh)
        il = dcfg.intermediate_size // tp
        self.layers = []
        for l in range(dcfg.num_hidden_layers):
            p = f"layers.{l}."
            wq = get(p + "self_attn.q_proj.weight")[r * hl * Dh:(r + 1) * hl * Dh]
            wk = get(p + "self_attn.k_proj.weight").view(dcfg.num_key_value_heads, Dh, H)[kv_heads].reshape(-1, H)
            wv = get(p + "self_attn.v_proj.weight").view(dcfg.num_key_value_heads, Dh, H)[kv_heads].reshape(-1, H)
            g = get(p + "mlp.gate_proj.weight")[r * il:(r + 1) * il]
            u = get(p + "mlp.up_proj.weight")[r * il:(r + 1) * il]
            gu = torch.stack([g.reshape(il // GU_BLOCK, GU_BLOCK, H), u.reshape(il // GU_BLOCK, GU_BLOCK, H)], 1)
            self.layers.append(dict(
                w_qkv=pw(torch.cat([wq, wk, wv], 0).contiguous()),
                w_kv=pw(torch.cat([wk, wv], 0).contiguous()),
                w_o=pw(get(p + "self_attn.o_proj.weight")[:, r * hl * Dh:(r + 1) * hl * Dh].contiguous()),
                qn=f32(p + "self_attn.q_norm.weight"), kn=f32(p + "self_attn.k_norm.weight"),
                in_norm=f32(p + "input_layernorm.weight"), post_norm=f32(p + "post_attention_layernorm.weight"),
                w_gu=pw(gu.reshape(2 * il, H).contiguous()),
                w_down=pw(get(p + "mlp.down_proj.weight")[:, r * il:(r + 1) * il].contiguous()),
                # [4 * H / group, H] dynamic-kernel projections (replicated) and [phase, tap, H] bases
                w_aconv=pw(get(p + "attention_conv.kernel_projection.weight").contiguous()),
                b_aconv=f32(p + "attention_conv.base_kernel"),
                w_mconv=pw(get(p + "mlp_conv.kernel_projection.weight").contiguous()),
                b_mconv=f32(p + "mlp_conv.base_kernel"),
            ))
        self.w_sel = pw(get("candidate_selector.hidden_projection.weight").contiguous())     # [rank, H]
        self.pred = get("candidate_selector.predecessor_codebook").contiguous()              # [V, rank]
        self.succ = get("candidate_selector.successor_codebook").contiguous()
        # plain rotary table over the whole head
        self.inv_freq = (1.0 / (dcfg.rope_theta ** (torch.arange(0, Dh, 2, dtype=torch.float32) / Dh))).to(dev)
        self.rope_scale = 1.0
        self.max_context = max_context or target.rt.max_context
        cap = self.max_context + 2 * dcfg.block_rows
        self.slots = slots
        self.kctx_all = torch.zeros(slots, dcfg.num_hidden_layers, cap, kvl, Dh, device=dev, dtype=dt)
        self.vctx_all = torch.zeros(slots, dcfg.num_hidden_layers, cap, kvl, Dh, device=dev, dtype=dt)
        self.positions = [0] * slots
        self.use_graphs = target.use_graphs
        self._graphs = {}
        self._init_propose_buffers(dcfg.block_rows)

    def history_floor(self, pos: int) -> int:
        """Lowest history row a block at ``pos`` or later can still see: older rows are masked for
        good, so a prefix checkpoint need not keep them (rows below it only have to stay finite,
        which every row ever written or zero-initialised is)."""
        return max(0, pos - self.window)

    # -------------------------------------------------------------------------------- propose
    def _branch_open(self, h, norm_w, w_kernel, base):
        """RMSNorm, the branch's dynamic kernels and its opening convolution -> (bf16 rows, kernels)."""
        n = self.ops.rms_norm(h, norm_w, self.eps, self.dtype)
        kern = self.ops.linear(n, w_kernel)
        return self.ops.draft_conv(n, kern, 0, base[0], self.group, out_dtype=self.dtype), kern

    @torch.no_grad()
    def forward_block(self, anchor: torch.Tensor, positions: torch.Tensor | None = None, slot: int = 0):
        """Block forward at the history frontier; returns (local-vocab logits [R, V_l] fp32,
        selector features [R, rank] bf16)."""
        R, pos = self.rows, self.positions[slot]
        ids = torch.full((R,), self.mask_id, dtype=torch.long, device=self.device)
        ids[:1] = anchor.reshape(1)
        h = self.ops.embedding(ids, self.target.embed).float()
        if positions is None:
            positions = torch.arange(pos, pos + R, device=self.device, dtype=torch.int32)
        for l, L in enumerate(self.layers):
            x, kern = self._branch_open(h, L["in_norm"], L["w_aconv"], L["b_aconv"])
            qkv = self.ops.linear(x, L["w_qkv"])
            o = self.ops.draft_block_attention(qkv, L["qn"], L["kn"], self.inv_freq, self.rope_scale, self.heads,
                                               self.eps, positions, self.kctx_all[slot, l], self.vctx_all[slot, l],
                                               self.dtype, window=self.window)
            self.ops.draft_conv(self._row_par(o, L["w_o"]), kern, 2, L["b_aconv"][1], self.group, residual=h)
            x, kern = self._branch_open(h, L["post_norm"], L["w_mconv"], L["b_mconv"])
            gu = self.ops.linear_swiglu(x, L["w_gu"], GU_BLOCK)
            self.ops.draft_conv(self._row_par(gu, L["w_down"]), kern, 2, L["b_mconv"][1], self.group, residual=h)
        hn = self.ops.rms_norm(h, self.norm, self.eps, self.dtype)
        logits = self.ops.linear(hn, self.target.lm_head, out_dtype=torch.float32)
        return logits, self.ops.linear(hn, self.w_sel)

    def candidates(self, logits: torch.Tensor):
        """Top ``candidates`` (global ids, logits) per row over the whole vocabulary: each rank's
        top entries, gathered, ordered by logit with ties to the lower id
        (``scripts/ci/draft_shared_head.py:41-68``)."""
        v, i = torch.topk(logits, self.n_cand, dim=-1)
        i = i + self.target.vocab_offset
        if self.tp > 1:
            v = self.comm.all_gather_cat(v.contiguous(), 1)
            i = self.comm.all_gather_cat(i.contiguous(), 1)
        o = torch.argsort(i, dim=-1, stable=True)
        v, i = v.gather(-1, o), i.gather(-1, o)
        o = torch.argsort(v, dim=-1, descending=True, stable=True)[:, :self.n_cand]
        return i.gather(-1, o).contiguous(), v.gather(-1, o).contiguous()

    def _propose_eager(self, anchor, positions=None, slot: int = 0):
        logits, feats = self.forward_block(anchor, positions, slot)
        cand, unary = self.candidates(logits)
        return self.ops.draft_select(feats, cand, unary, anchor, self.pred, self.succ)
