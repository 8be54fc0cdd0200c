"""DFlash block drafter with the swappable-objective hook.

Interface-compatible with harvestingmoon/cuda-spec-decode
models/dflash/model.py: same class names, constructor arguments, parameter
names (so state dicts load either way), attention mask rule and the
``compute_loss(target_features, ground_truth_block_tokens, loss_fn=None)``
hook (model.py:152-170) that lets the fused losses of this library replace
plain cross entropy.

Architecture (model.py:76-150): target features -> proj_in -> append
``block_size`` trainable slot queries -> pre-RMSNorm transformer layers under
a mask where context tokens are causal and block tokens see every token ->
RMSNorm -> proj_out -> optional RMSNorm -> frozen verifier lm_head ->
[batch, block_size, V] logits. The mask is applied by its structure (the
context causal, the block queries over every token), never as a [T, T]
tensor. Layers on this library's kernels (specdec.drafter): the RMSNorms
(fp32 or bf16 activations) and, for bf16 q/k/v with 64-dim heads (e.g.
under bf16 autocast), the attention forward on the tensor cores; otherwise
attention runs through F.scaled_dot_product_attention (a causal attention
over the context plus an unmasked one for the block queries). GEMMs are
cuBLAS (nn.Linear).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from specdec import drafter as _kernels


class RMSNorm(nn.RMSNorm):
    """torch.nn.RMSNorm (same parameters and state-dict keys) whose forward
    runs the library's RMSNorm kernels on CUDA tensors."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if len(self.normalized_shape) == 1 and _kernels.rms_norm_supported(x, self.weight):
            return _kernels.rms_norm(x, self.weight, self.eps)
        return super().forward(x)


class DFlashAttention(nn.Module):
    """Multi-head attention taking an additive mask (reference model.py:25-53)."""

    def __init__(self, d_model: int, num_heads: int, qkv_bias: bool = False):
        super().__init__()
        if d_model % num_heads:
            raise AssertionError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.q_proj = nn.Linear(d_model, d_model, bias=qkv_bias)
        self.k_proj = nn.Linear(d_model, d_model, bias=qkv_bias)
        self.v_proj = nn.Linear(d_model, d_model, bias=qkv_bias)
        self.out_proj = nn.Linear(d_model, d_model, bias=qkv_bias)

    def _heads(self, t: torch.Tensor) -> torch.Tensor:
        b, s, _ = t.shape
        return t.view(b, s, self.num_heads, self.head_dim).transpose(1, 2)

    def forward(self, x: torch.Tensor, attn_mask: torch.Tensor | None = None,
                n_ctx: int | None = None) -> torch.Tensor:
        """attn_mask: additive [.., T, T] mask (the reference's form). n_ctx
        instead states the DFlash mask by its structure -- the first n_ctx
        tokens causal among themselves and blind to the rest, the others
        seeing every token -- and runs it as two mask-free attentions (causal
        over the context; the block queries over all keys), which the fused
        SDPA kernels handle without reading a [T, T] mask."""
        b, s, _ = x.shape
        if n_ctx is not None and attn_mask is None:
            qs = self.q_proj(x).view(b, s, self.num_heads, self.head_dim)
            if _kernels.attention_supported(qs):  # [b, s, heads, dim]: the kernels' layout
                ks = self.k_proj(x).view(b, s, self.num_heads, self.head_dim)
                vs = self.v_proj(x).view(b, s, self.num_heads, self.head_dim)
                y = _kernels.dflash_attention(qs, ks.to(qs.dtype), vs.to(qs.dtype), n_ctx)
                return self.out_proj(y.reshape(b, s, self.d_model))
        q, k, v = self._heads(self.q_proj(x)), self._heads(self.k_proj(x)), self._heads(self.v_proj(x))
        if n_ctx is not None and attn_mask is None:
            y_ctx = F.scaled_dot_product_attention(q[:, :, :n_ctx], k[:, :, :n_ctx], v[:, :, :n_ctx],
                                                   is_causal=True)
            y_blk = F.scaled_dot_product_attention(q[:, :, n_ctx:], k, v)
            y = torch.cat([y_ctx, y_blk], dim=2)
        else:
            mask = None if attn_mask is None else attn_mask.to(q.dtype)
            y = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return self.out_proj(y.transpose(1, 2).reshape(b, s, self.d_model))


class DFlashTransformerLayer(nn.Module):
    """Pre-norm block: x + attn(norm(x)), then x + mlp(norm(x)) (reference model.py:56-73)."""

    def __init__(self, d_model: int, num_heads: int, d_ffn: int):
        super().__init__()
        self.norm1 = RMSNorm(d_model)
        self.attn = DFlashAttention(d_model=d_model, num_heads=num_heads)
        self.norm2 = RMSNorm(d_model)
        self.mlp = nn.Sequential(nn.Linear(d_model, d_ffn, bias=False), nn.SiLU(),
                                 nn.Linear(d_ffn, d_model, bias=False))

    def forward(self, x: torch.Tensor, attn_mask: torch.Tensor | None = None,
                n_ctx: int | None = None) -> torch.Tensor:
        x = x + self.attn(self.norm1(x), attn_mask=attn_mask, n_ctx=n_ctx)
        return x + self.mlp(self.norm2(x))


class DFlashSpeculator(nn.Module):
    """Block-parallel drafter emitting ``block_size`` draft logits per sequence."""

    def __init__(self, d_target: int, d_model: int, target_vocab_size: int, block_size: int = 4,
                 num_layers: int = 3, num_heads: int = 4,
                 target_lm_head: nn.Linear | None = None, norm_before_head: bool = True):
        super().__init__()
        self.d_target = d_target
        self.d_model = d_model
        self.block_size = block_size
        self.target_vocab_size = target_vocab_size
        self.proj_in = nn.Linear(d_target, d_model, bias=False)
        self.slot_queries = nn.Parameter(0.02 * torch.randn(1, block_size, d_model))
        self.layers = nn.ModuleList(
            DFlashTransformerLayer(d_model, num_heads, 4 * d_model) for _ in range(num_layers))
        self.norm_out = RMSNorm(d_model)
        self.proj_out = nn.Linear(d_model, d_target, bias=False)
        self.final_norm = RMSNorm(d_target) if norm_before_head else None
        if target_lm_head is not None:
            self.lm_head = target_lm_head
            self.lm_head.weight.requires_grad = False  # the verifier head stays frozen
        else:
            self.lm_head = nn.Linear(d_target, target_vocab_size, bias=False)

    def _build_dflash_mask(self, S_ctx: int, S_block: int, device) -> torch.Tensor:
        """Additive [1, 1, T, T] mask: context rows causal over the context and
        blind to the block; block rows see every token."""
        T = S_ctx + S_block
        row = torch.arange(T, device=device).view(T, 1)
        col = torch.arange(T, device=device).view(1, T)
        visible = (row >= S_ctx) | ((col <= row) & (col < S_ctx))
        mask = torch.zeros(T, T, device=device)
        mask.masked_fill_(~visible, float("-inf"))
        return mask.view(1, 1, T, T)

    def forward(self, target_features: torch.Tensor) -> torch.Tensor:
        """target_features [batch, S_ctx, d_target] -> draft logits [batch, block_size, V]."""
        b, s_ctx, _ = target_features.shape
        h = torch.cat([self.proj_in(target_features),
                       self.slot_queries.expand(b, -1, -1).to(target_features.dtype)], dim=1)
        # the _build_dflash_mask rule, applied by structure (no [T, T] mask tensor)
        for layer in self.layers:
            h = layer(h, n_ctx=s_ctx)
        feat = self.proj_out(self.norm_out(h)[:, s_ctx:, :])
        if self.final_norm is not None:
            feat = self.final_norm(feat)
        return self.lm_head(feat)

    def compute_loss(self, target_features: torch.Tensor, ground_truth_block_tokens: torch.Tensor,
                     loss_fn=None) -> torch.Tensor:
        """Training loss over the block slots. ``loss_fn(logits, targets) -> scalar``
        swaps the objective (dpace_loss, dflash_objective(...)); None = plain CE."""
        logits = self.forward(target_features)
        if loss_fn is not None:
            return loss_fn(logits, ground_truth_block_tokens)
        return F.cross_entropy(logits.reshape(-1, self.target_vocab_size),
                               ground_truth_block_tokens.reshape(-1))

    @torch.no_grad()
    def draft(self, target_features: torch.Tensor):
        """Single-pass drafting: (draft_tokens [batch, block], draft_logits)."""
        logits = self.forward(target_features)
        return logits.argmax(dim=-1), logits
