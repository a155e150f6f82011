"""Drop-in tropical transformer layers and models (tropformer_dropin.py).

Mirrors the public classes of tropformer_dropin.py -- same constructors,
parameter names and state-dict keys, PyTorch-style ``forward`` signatures --
with the tropical parts on this library's kernels:

* ``TropicalLinear`` (tropformer_dropin.py:45-79): the max-plus GEMM, STE
  backward in training, argmax backward in eval (the class of tropical.py;
  the math of both reference files is the same);
* the tropical attention score ``max_f(Q + K) * d_k^-1/2`` of
  ``TropicalMultiHeadAttention`` (:167-285, score at :236-240): the batched
  strided max-plus kernel over the [B, H, L, d_k] head views, with the argmax
  scatter backward that autograd of ``.max(-1)`` gives (value-only kernel
  when no gradient is taken), also across a ``TropicalKVCache``;
* ``TropicalHybridFFN`` (:288-328): in inference ``lf_act(trop_up(x))`` is one
  kernel (the LF activation fused into the max-plus epilogue).

Everything else (projections, gate, masks, Maslov softmax, layer norms,
residuals, embeddings) is the reference's PyTorch expression.  The encoder /
decoder layers, stacks and models below only compose these, as the reference
ones do; alternatively swap ``TropicalLinear``, ``TropicalMultiHeadAttention``
and ``TropicalHybridFFN`` into the reference module before building a model.
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from . import tropical
from .tropical import MaslovTemperature, TropicalLinear

__all__ = [
    "TropicalLinear", "MaslovTemperature", "LFDualActivation", "TropicalKVCache",
    "TropicalMultiHeadAttention", "TropicalHybridFFN", "TropicalEncoderLayer",
    "TropicalDecoderLayer", "TropicalEncoder", "TropicalDecoder", "TropicalTransformer",
    "TropicalEncoderModel", "TropicalDecoderModel", "TropicalViT",
    "TropicalViTForClassification", "make_causal_mask", "maslov_summary", "lf_blend_summary",
]


class LFDualActivation(tropical.LFDualActivation):
    """Tropical polynomial activation and its Legendre-Fenchel dual
    (tropformer_dropin.py:100-140); "blend" is this file's default mode."""

    def __init__(self, dim: int, num_pieces: int = 8, mode: str = "blend"):
        super().__init__(dim, num_pieces=num_pieces, mode=mode)


@dataclass
class TropicalKVCache:
    """Keys and values of earlier decoding steps (tropformer_dropin.py:143-164);
    new ones are appended along the sequence axis (dim 2 of [B, H, L, d_k])."""

    k: Optional[torch.Tensor] = None
    v: Optional[torch.Tensor] = None

    def update(self, k_new: torch.Tensor, v_new: torch.Tensor):
        if self.k is None:
            self.k, self.v = k_new, v_new
        else:
            self.k = torch.cat([self.k, k_new], dim=2)
            self.v = torch.cat([self.v, v_new], dim=2)
        return self.k, self.v

    def reset(self):
        self.k = self.v = None


def _grad_needed(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


class TropicalMultiHeadAttention(nn.Module):
    """Self- or cross-attention blending tropical and classical scores
    (tropformer_dropin.py:167-285): ``g * trop + (1 - g) * classical`` with a
    sigmoid gate from the queries (cross: from the mean query and key
    contexts), additive and padding masks, Maslov softmax, @V, out_proj."""

    def __init__(self, d_model: int, num_heads: int, dropout: float = 0.1,
                 init_temp: float = 1.0, is_cross_attention: bool = False):
        super().__init__()
        assert d_model % num_heads == 0
        self.d_model = d_model
        self.num_heads = num_heads
        self.d_k = d_model // num_heads
        self._scale = self.d_k ** -0.5
        self.is_cross_attention = is_cross_attention
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.score_gate = nn.Linear((2 if is_cross_attention else 1) * d_model, num_heads)
        nn.init.zeros_(self.score_gate.weight)
        nn.init.constant_(self.score_gate.bias, -2.0)
        self.maslov = MaslovTemperature(num_heads, init_temp)
        self.attn_dropout = nn.Dropout(dropout)

    def _split_heads(self, x: torch.Tensor) -> torch.Tensor:
        B, L, _ = x.shape
        return x.view(B, L, self.num_heads, self.d_k).transpose(1, 2)

    def _tropical_scores(self, Q: torch.Tensor, K: torch.Tensor) -> torch.Tensor:
        if _grad_needed(Q, K):
            return ops.TropicalScoreFunction.apply(Q, K, self._scale, None)
        return ops.tropical_scores(Q, K, self._scale, argmax=False)[0]

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                attn_mask: Optional[torch.Tensor] = None,
                key_padding_mask: Optional[torch.Tensor] = None,
                cache: Optional[TropicalKVCache] = None, need_weights: bool = False):
        B, L_q, D = query.shape
        Q = self._split_heads(self.q_proj(query))
        K = self._split_heads(self.k_proj(key))
        V = self._split_heads(self.v_proj(value))
        if cache is not None:
            K, V = cache.update(K, V)
        class_scores = torch.matmul(Q, K.transpose(-2, -1)) * self._scale
        trop_scores = self._tropical_scores(Q, K)
        if self.is_cross_attention:
            ctx = torch.cat([query.mean(dim=1), key.mean(dim=1)], dim=-1)
            g = torch.sigmoid(self.score_gate(ctx))[:, :, None, None]          # (B, H, 1, 1)
        else:
            g = torch.sigmoid(self.score_gate(query)).permute(0, 2, 1)[..., None]  # (B, H, Lq, 1)
        scores = g * trop_scores + (1.0 - g) * class_scores
        if attn_mask is not None:
            if attn_mask.dim() == 2:
                scores = scores + attn_mask[None, None]
            elif attn_mask.dim() == 3:
                scores = scores + attn_mask[:, None]
            else:
                scores = scores + attn_mask
        if key_padding_mask is not None:
            scores = scores.masked_fill(key_padding_mask[:, None, None, :], -1e9)
        attn = self.attn_dropout(self.maslov(scores))
        out = torch.matmul(attn, V).transpose(1, 2).contiguous().view(B, L_q, D)
        return self.out_proj(out), (attn if need_weights else None)


class TropicalHybridFFN(nn.Module):
    """Tropical branch (TropicalLinear -> LFDualActivation -> dropout) and
    classical branch (Linear -> GELU) fused by sigmoid(gate_proj(x)), then
    down_proj and dropout (tropformer_dropin.py:288-328; no norm or residual)."""

    def __init__(self, d_model: int, ffn_dim: int, dropout: float = 0.1,
                 lf_pieces: int = 8, lf_mode: str = "blend"):
        super().__init__()
        self.trop_up = TropicalLinear(d_model, ffn_dim)
        self.lf_act = LFDualActivation(ffn_dim, num_pieces=lf_pieces, mode=lf_mode)
        self.trop_drop = nn.Dropout(dropout)
        self.class_up = nn.Linear(d_model, ffn_dim)
        self.gelu = nn.GELU()
        self.gate_proj = nn.Linear(d_model, ffn_dim)
        nn.init.zeros_(self.gate_proj.weight)
        nn.init.constant_(self.gate_proj.bias, -2.0)
        self.down_proj = nn.Linear(ffn_dim, d_model)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        trop = self.trop_drop(tropical.tropical_up_lf(self.trop_up, self.lf_act, x))
        classical = self.gelu(self.class_up(x))
        g = torch.sigmoid(self.gate_proj(x))
        return self.dropout(self.down_proj(g * trop + (1.0 - g) * classical))


class TropicalEncoderLayer(nn.Module):
    """Drop-in for nn.TransformerEncoderLayer (tropformer_dropin.py:331-403):
    forward(src, src_mask=None, src_key_padding_mask=None); pre-norm by default."""

    def __init__(self, d_model: int, nhead: int, dim_feedforward: int = 2048,
                 dropout: float = 0.1, lf_pieces: int = 8, lf_mode: str = "blend",
                 init_temp: float = 1.0, batch_first: bool = True, norm_first: bool = True):
        super().__init__()
        self.batch_first = batch_first
        self.norm_first = norm_first
        self.self_attn = TropicalMultiHeadAttention(d_model, nhead, dropout=dropout,
                                                    init_temp=init_temp)
        self.ffn = TropicalHybridFFN(d_model, dim_feedforward, dropout=dropout,
                                     lf_pieces=lf_pieces, lf_mode=lf_mode)
        self.norm1 = nn.LayerNorm(d_model)
        self.norm2 = nn.LayerNorm(d_model)
        self.dropout1 = nn.Dropout(dropout)
        self.dropout2 = nn.Dropout(dropout)

    def forward(self, src: torch.Tensor, src_mask: Optional[torch.Tensor] = None,
                src_key_padding_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        x = src if self.batch_first else src.transpose(0, 1)
        masks = dict(attn_mask=src_mask, key_padding_mask=src_key_padding_mask)
        if self.norm_first:
            h = self.norm1(x)
            x = x + self.dropout1(self.self_attn(h, h, h, **masks)[0])
            x = x + self.dropout2(self.ffn(self.norm2(x)))
        else:
            x = self.norm1(x + self.dropout1(self.self_attn(x, x, x, **masks)[0]))
            x = self.norm2(x + self.dropout2(self.ffn(x)))
        return x if self.batch_first else x.transpose(0, 1)


class TropicalDecoderLayer(nn.Module):
    """Drop-in for nn.TransformerDecoderLayer (tropformer_dropin.py:406-492):
    self-attention, cross-attention over ``memory``, hybrid FFN."""

    def __init__(self, d_model: int, nhead: int, dim_feedforward: int = 2048,
                 dropout: float = 0.1, lf_pieces: int = 8, lf_mode: str = "blend",
                 init_temp: float = 1.0, batch_first: bool = True, norm_first: bool = True):
        super().__init__()
        self.batch_first = batch_first
        self.norm_first = norm_first
        self.self_attn = TropicalMultiHeadAttention(d_model, nhead, dropout=dropout,
                                                    init_temp=init_temp)
        self.cross_attn = TropicalMultiHeadAttention(d_model, nhead, dropout=dropout,
                                                     init_temp=init_temp, is_cross_attention=True)
        self.ffn = TropicalHybridFFN(d_model, dim_feedforward, dropout=dropout,
                                     lf_pieces=lf_pieces, lf_mode=lf_mode)
        self.norm1 = nn.LayerNorm(d_model)
        self.norm2 = nn.LayerNorm(d_model)
        self.norm3 = nn.LayerNorm(d_model)
        self.dropout1 = nn.Dropout(dropout)
        self.dropout2 = nn.Dropout(dropout)
        self.dropout3 = nn.Dropout(dropout)

    def forward(self, tgt: torch.Tensor, memory: torch.Tensor,
                tgt_mask: Optional[torch.Tensor] = None,
                memory_mask: Optional[torch.Tensor] = None,
                tgt_key_padding_mask: Optional[torch.Tensor] = None,
                memory_key_padding_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not self.batch_first:
            tgt, memory = tgt.transpose(0, 1), memory.transpose(0, 1)
        x = tgt
        self_masks = dict(attn_mask=tgt_mask, key_padding_mask=tgt_key_padding_mask)
        mem_masks = dict(attn_mask=memory_mask, key_padding_mask=memory_key_padding_mask)
        if self.norm_first:
            h = self.norm1(x)
            x = x + self.dropout1(self.self_attn(h, h, h, **self_masks)[0])
            h = self.norm2(x)
            x = x + self.dropout2(self.cross_attn(h, memory, memory, **mem_masks)[0])
            x = x + self.dropout3(self.ffn(self.norm3(x)))
        else:
            x = self.norm1(x + self.dropout1(self.self_attn(x, x, x, **self_masks)[0]))
            x = self.norm2(x + self.dropout2(self.cross_attn(x, memory, memory, **mem_masks)[0]))
            x = self.norm3(x + self.dropout3(self.ffn(x)))
        return x if self.batch_first else x.transpose(0, 1)


class TropicalEncoder(nn.Module):
    """Stack of copies of an encoder layer, optional final norm
    (tropformer_dropin.py:495-515)."""

    def __init__(self, encoder_layer: TropicalEncoderLayer, num_layers: int,
                 norm: Optional[nn.Module] = None):
        super().__init__()
        self.layers = nn.ModuleList([copy.deepcopy(encoder_layer) for _ in range(num_layers)])
        self.norm = norm

    def forward(self, src: torch.Tensor, mask: Optional[torch.Tensor] = None,
                src_key_padding_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = src
        for layer in self.layers:
            out = layer(out, src_mask=mask, src_key_padding_mask=src_key_padding_mask)
        return self.norm(out) if self.norm is not None else out


class TropicalDecoder(nn.Module):
    """Stack of copies of a decoder layer, optional final norm
    (tropformer_dropin.py:518-546)."""

    def __init__(self, decoder_layer: TropicalDecoderLayer, num_layers: int,
                 norm: Optional[nn.Module] = None):
        super().__init__()
        self.layers = nn.ModuleList([copy.deepcopy(decoder_layer) for _ in range(num_layers)])
        self.norm = norm

    def forward(self, tgt: torch.Tensor, memory: torch.Tensor,
                tgt_mask: Optional[torch.Tensor] = None,
                memory_mask: Optional[torch.Tensor] = None,
                tgt_key_padding_mask: Optional[torch.Tensor] = None,
                memory_key_padding_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = tgt
        for layer in self.layers:
            out = layer(out, memory, tgt_mask=tgt_mask, memory_mask=memory_mask,
                        tgt_key_padding_mask=tgt_key_padding_mask,
                        memory_key_padding_mask=memory_key_padding_mask)
        return self.norm(out) if self.norm is not None else out


class TropicalTransformer(nn.Module):
    """Encoder-decoder drop-in for nn.Transformer (tropformer_dropin.py:549-613)."""

    def __init__(self, d_model: int = 512, nhead: int = 8, num_encoder_layers: int = 6,
                 num_decoder_layers: int = 6, dim_feedforward: int = 2048, dropout: float = 0.1,
                 lf_pieces: int = 8, lf_mode: str = "blend", init_temp: float = 1.0,
                 batch_first: bool = True, norm_first: bool = True):
        super().__init__()
        args = (d_model, nhead, dim_feedforward, dropout, lf_pieces, lf_mode, init_temp,
                batch_first, norm_first)
        self.encoder = TropicalEncoder(TropicalEncoderLayer(*args), num_encoder_layers,
                                       norm=nn.LayerNorm(d_model) if norm_first else None)
        self.decoder = TropicalDecoder(TropicalDecoderLayer(*args), num_decoder_layers,
                                       norm=nn.LayerNorm(d_model) if norm_first else None)
        self.d_model = d_model
        self.nhead = nhead
        self.batch_first = batch_first

    def forward(self, src: torch.Tensor, tgt: torch.Tensor,
                src_mask: Optional[torch.Tensor] = None, tgt_mask: Optional[torch.Tensor] = None,
                memory_mask: Optional[torch.Tensor] = None,
                src_key_padding_mask: Optional[torch.Tensor] = None,
                tgt_key_padding_mask: Optional[torch.Tensor] = None,
                memory_key_padding_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        memory = self.encoder(src, mask=src_mask, src_key_padding_mask=src_key_padding_mask)
        return self.decoder(tgt, memory, tgt_mask=tgt_mask, memory_mask=memory_mask,
                            tgt_key_padding_mask=tgt_key_padding_mask,
                            memory_key_padding_mask=memory_key_padding_mask)


def make_causal_mask(seq_len: int, device: torch.device) -> torch.Tensor:
    """Additive causal mask, -1e9 above the diagonal (tropformer_dropin.py:723-733;
    a finite tropical zero keeps the max-plus score free of -inf)."""
    return torch.triu(torch.full((seq_len, seq_len), -1e9, device=device), diagonal=1)


class _TokenModel(nn.Module):
    # token + learned position embeddings scaled by sqrt(d_model), then an
    # encoder stack with a final norm (the shared body of the two models below)
    def _body(self, vocab_size, d_model, nhead, num_layers, dim_feedforward, dropout,
              max_seq_len, lf_pieces, lf_mode, init_temp):
        self.d_model = d_model
        self.embed = nn.Embedding(vocab_size, d_model)
        self.pos_embed = nn.Embedding(max_seq_len, d_model)
        self.embed_drop = nn.Dropout(dropout)
        self.embed_scale = math.sqrt(d_model)
        layer = TropicalEncoderLayer(d_model, nhead, dim_feedforward, dropout, lf_pieces,
                                     lf_mode, init_temp)
        return TropicalEncoder(layer, num_layers, norm=nn.LayerNorm(d_model))

    def _embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        positions = torch.arange(input_ids.shape[1], device=input_ids.device)[None]
        return self.embed_drop(self.embed(input_ids) * self.embed_scale +
                               self.pos_embed(positions))


class TropicalEncoderModel(_TokenModel):
    """Encoder-only (BERT-style) model (tropformer_dropin.py:616-663); attention_mask
    1 = keep, 0 = padding."""

    def __init__(self, vocab_size: int, d_model: int = 512, nhead: int = 8, num_layers: int = 6,
                 dim_feedforward: int = 2048, dropout: float = 0.1, max_seq_len: int = 512,
                 lf_pieces: int = 8, lf_mode: str = "blend", init_temp: float = 1.0):
        super().__init__()
        self.encoder = self._body(vocab_size, d_model, nhead, num_layers, dim_feedforward,
                                  dropout, max_seq_len, lf_pieces, lf_mode, init_temp)

    def forward(self, input_ids: torch.Tensor,
                attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        pad = (attention_mask == 0) if attention_mask is not None else None
        return self.encoder(self._embed(input_ids), src_key_padding_mask=pad)


class TropicalDecoderModel(_TokenModel):
    """Decoder-only (GPT-style) causal language model (tropformer_dropin.py:665-720)."""

    def __init__(self, vocab_size: int, d_model: int = 512, nhead: int = 8, num_layers: int = 6,
                 dim_feedforward: int = 2048, dropout: float = 0.1, max_seq_len: int = 2048,
                 lf_pieces: int = 8, lf_mode: str = "blend", init_temp: float = 1.0):
        super().__init__()
        self.layers = self._body(vocab_size, d_model, nhead, num_layers, dim_feedforward,
                                 dropout, max_seq_len, lf_pieces, lf_mode, init_temp)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)

    def forward(self, input_ids: torch.Tensor,
                attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        mask = make_causal_mask(input_ids.shape[1], input_ids.device)
        pad = (attention_mask == 0) if attention_mask is not None else None
        x = self.layers(self._embed(input_ids), mask=mask, src_key_padding_mask=pad)
        return self.lm_head(x)


class TropicalViT(nn.Module):
    """Vision transformer on a tropical encoder (tropformer_dropin.py:739-797):
    patchify -> linear embedding -> CLS + learned positions -> encoder -> norm."""

    def __init__(self, img_size: int = 224, patch_size: int = 16, in_channels: int = 3,
                 d_model: int = 768, nhead: int = 12, num_layers: int = 12,
                 dim_feedforward: int = 3072, dropout: float = 0.1, lf_pieces: int = 8,
                 lf_mode: str = "blend", init_temp: float = 1.0):
        super().__init__()
        assert img_size % patch_size == 0
        self.patch_size = patch_size
        num_patches = (img_size // patch_size) ** 2
        self.patch_embed = nn.Linear(in_channels * patch_size * patch_size, d_model)
        nn.init.trunc_normal_(self.patch_embed.weight, std=0.02)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, d_model))
        self.pos_embed = nn.Parameter(torch.zeros(1, num_patches + 1, d_model))
        nn.init.trunc_normal_(self.cls_token, std=0.02)
        nn.init.trunc_normal_(self.pos_embed, std=0.02)
        self.embed_drop = nn.Dropout(dropout)
        layer = TropicalEncoderLayer(d_model, nhead, dim_feedforward, dropout, lf_pieces,
                                     lf_mode, init_temp)
        self.encoder = TropicalEncoder(layer, num_layers, norm=nn.LayerNorm(d_model))

    def patchify(self, x: torch.Tensor) -> torch.Tensor:
        B, C, H, W = x.shape
        p = self.patch_size
        x = x.view(B, C, H // p, p, W // p, p).permute(0, 2, 4, 1, 3, 5).contiguous()
        return x.view(B, -1, C * p * p)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.patch_embed(self.patchify(x))
        x = torch.cat([self.cls_token.expand(x.shape[0], -1, -1), x], dim=1)
        return self.encoder(self.embed_drop(x + self.pos_embed))


class TropicalViTForClassification(nn.Module):
    """TropicalViT plus a linear head on the CLS token (tropformer_dropin.py:800-819)."""

    def __init__(self, num_classes: int = 10, **vit_kwargs):
        super().__init__()
        self.vit = TropicalViT(**vit_kwargs)
        self.head = nn.Linear(vit_kwargs.get("d_model", 768), num_classes)
        nn.init.zeros_(self.head.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.head(self.vit(x)[:, 0])

    def count_params(self) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad)


def maslov_summary(model: nn.Module) -> dict:
    """Per-head Maslov temperatures of every MaslovTemperature in ``model``."""
    return {name: m.temperatures.detach().cpu() for name, m in model.named_modules()
            if isinstance(m, tropical.MaslovTemperature)}


def lf_blend_summary(model: nn.Module) -> dict:
    """Mean sigmoid(blend_gate) of every blending LFDualActivation in ``model``."""
    return {name: torch.sigmoid(m.blend_gate).detach().cpu().mean().item()
            for name, m in model.named_modules()
            if isinstance(m, tropical.LFDualActivation) and hasattr(m, "blend_gate")}
