"""Torch-CPU restatement of the Qwen2 decoder forward on the reference's path.

Op-for-op the same sequence as ``transformers`` 5.5.0
``models/qwen2/modeling_qwen2.py`` so that, on the CPU, it reproduces
``Qwen2ForCausalLM`` bit for bit:

* ``Qwen2RMSNorm.forward`` (:258-263);
* ``Qwen2RotaryEmbedding.compute_default_rope_parameters`` / ``forward`` (:89-113),
  ``rotate_half`` / ``apply_rotary_pos_emb`` (:116-146);
* ``Qwen2Attention.forward`` (:214-245) with ``sdpa_attention_forward``
  (``integrations/sdpa_attention.py:40-104``): causal SDPA with
  ``enable_gqa`` for the prefill, and for decode the reference's
  ``folded_sdpa`` (``rapidtinyrec/folded_attention.py:16-31``) which packs the
  query heads of each KV head into rows;
* ``Qwen2MLP.forward`` (:46-48), ``Qwen2DecoderLayer.forward`` (:290-309);
* last-token LM head (``logits_to_keep=1``).

The KV layout matches the reference's shared prefill: one ``[1,Hkv,L,D]``
prefix per layer (``prefix_prefill.py:56-59``) and per-beam suffix rows that
are concatenated behind the expanded prefix (``shared_prefix.py:22-29``), which
is numerically the dense ``batch_repeat_interleave`` cache of ``PrefillOnce``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x, weight, eps):
    input_dtype = x.dtype
    h = x.to(torch.float32)
    variance = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    return weight * h.to(input_dtype)


def rope_inv_freq(head_dim, theta):
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))


def rope_cos_sin(inv_freq, position_ids, dtype):
    """``position_ids [B, S]`` -> cos/sin ``[B, S, D]`` exactly as HF computes them."""
    inv = inv_freq[None, :, None].float().expand(position_ids.shape[0], -1, 1)
    pos = position_ids[:, None, :].float()
    freqs = (inv.float() @ pos.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return (emb.cos() * 1.0).to(dtype), (emb.sin() * 1.0).to(dtype)


def rope_table(head_dim, theta, n_positions):
    """cos/sin ``[n_positions, head_dim // 2]`` float32 - the table the CUDA path uploads.

    Built from HF's per-call computation for blocks of positions small enough
    that torch evaluates each on one thread (every element vectorised), which is
    how HF evaluates a prompt of up to 256 positions.
    """
    inv = rope_inv_freq(head_dim, theta)
    rows = max(1, 16384 // head_dim)
    parts = [rope_cos_sin(inv, torch.arange(i, min(i + rows, n_positions))[None, :], torch.float32)
             for i in range(0, n_positions, rows)]
    cos = torch.cat([c for c, _ in parts], dim=1)
    sin = torch.cat([s for _, s in parts], dim=1)
    return cos[0, :, :head_dim // 2].contiguous(), sin[0, :, :head_dim // 2].contiguous()


def rotate_half(x):
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(q, k, cos, sin):
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


class Qwen2Oracle:
    """Forward passes over a shared prefix and per-beam suffixes.

    ``weights`` uses the Hugging Face Qwen2 state-dict names.
    """

    def __init__(self, cfg, weights, dtype=torch.float32, fold=True):
        self.cfg = cfg
        self.dtype = dtype
        self.fold = fold
        self.w = {k: v.detach().to(device='cpu', dtype=dtype) for k, v in weights.items()}
        if 'lm_head.weight' not in self.w:
            self.w['lm_head.weight'] = self.w['model.embed_tokens.weight']
        # ``model.to(dtype)`` also casts the non-persistent ``inv_freq`` buffer,
        # so a BF16 model rotates with bf16-rounded frequencies.
        self.inv_freq = rope_inv_freq(cfg.head_dim, cfg.rope_theta).to(dtype).float()
        self.scaling = cfg.head_dim ** -0.5

    def _attention(self, n, h, cos, sin, cache, decode):
        cfg, w = self.cfg, self.w
        p = f'model.layers.{n}.self_attn.'
        bsz, q_len = h.shape[:2]
        shape = (bsz, q_len, -1, cfg.head_dim)
        q = F.linear(h, w[p + 'q_proj.weight'], w[p + 'q_proj.bias']).view(shape).transpose(1, 2)
        k = F.linear(h, w[p + 'k_proj.weight'], w[p + 'k_proj.bias']).view(shape).transpose(1, 2)
        v = F.linear(h, w[p + 'v_proj.weight'], w[p + 'v_proj.bias']).view(shape).transpose(1, 2)
        q, k = apply_rope(q, k, cos, sin)
        if not decode:
            cache[n] = [k, v, None, None]
            out = F.scaled_dot_product_attention(q, k, v, attn_mask=None, dropout_p=0.0,
                                                 is_causal=q_len > 1, scale=self.scaling, enable_gqa=True)
        else:
            pk, pv, sk, sv = cache[n]
            sk = k if sk is None else torch.cat((sk, k), dim=-2)
            sv = v if sv is None else torch.cat((sv, v), dim=-2)
            cache[n][2], cache[n][3] = sk, sv
            keys = torch.cat((pk.expand(bsz, -1, -1, -1), sk), dim=-2)
            values = torch.cat((pv.expand(bsz, -1, -1, -1), sv), dim=-2)
            if self.fold and cfg.heads > cfg.kv_heads:
                packed = q.reshape(bsz, cfg.kv_heads, cfg.heads // cfg.kv_heads, cfg.head_dim)
                out = F.scaled_dot_product_attention(packed, keys, values, attn_mask=None, dropout_p=0.0,
                                                     is_causal=False, scale=self.scaling, enable_gqa=False)
                out = out.reshape(bsz, cfg.heads, 1, cfg.head_dim)
            else:
                out = F.scaled_dot_product_attention(q, keys, values, attn_mask=None, dropout_p=0.0,
                                                     is_causal=False, scale=self.scaling, enable_gqa=True)
        out = out.transpose(1, 2).contiguous().reshape(bsz, q_len, -1).contiguous()
        return F.linear(out, w[p + 'o_proj.weight'])

    def _forward(self, ids, positions, cache, decode):
        cfg, w = self.cfg, self.w
        x = F.embedding(ids, w['model.embed_tokens.weight'])
        cos, sin = rope_cos_sin(self.inv_freq, positions, x.dtype)
        for n in range(cfg.layers):
            p = f'model.layers.{n}.'
            residual = x
            h = rms_norm(x, w[p + 'input_layernorm.weight'], cfg.rms_eps)
            x = residual + self._attention(n, h, cos, sin, cache, decode)
            residual = x
            h = rms_norm(x, w[p + 'post_attention_layernorm.weight'], cfg.rms_eps)
            mlp = F.linear(F.silu(F.linear(h, w[p + 'mlp.gate_proj.weight'])) * F.linear(h, w[p + 'mlp.up_proj.weight']),
                           w[p + 'mlp.down_proj.weight'])
            x = residual + mlp
        x = rms_norm(x, w['model.norm.weight'], cfg.rms_eps)
        return F.linear(x[:, -1:, :], w['lm_head.weight'])

    @torch.inference_mode()
    def prefill(self, prompt_ids):
        """One row of ``L`` prompt tokens -> (logits ``[1, V]``, cache)."""
        ids = torch.as_tensor(prompt_ids, dtype=torch.long)[None, :]
        cache = [None] * self.cfg.layers
        positions = torch.arange(ids.shape[1])[None, :]
        return self._forward(ids, positions, cache, decode=False)[:, -1, :], cache

    @torch.inference_mode()
    def decode(self, tokens, position, cache):
        """``tokens [B]`` at ``position`` over ``cache`` -> logits ``[B, V]`` (cache updated)."""
        ids = torch.as_tensor(tokens, dtype=torch.long)[:, None]
        positions = torch.full_like(ids, position)
        return self._forward(ids, positions, cache, decode=True)[:, -1, :]

    @staticmethod
    def reorder(cache, beam_idx):
        """``_reorder_cache``: gather the suffix rows; the shared prefix is untouched."""
        for layer in cache:
            if layer[2] is not None:
                layer[2] = layer[2].index_select(0, beam_idx)
                layer[3] = layer[3].index_select(0, beam_idx)
