"""Steps of a Hugging Face Llama model through this library's fused layer
kernels, over the model's own weights and the engine's paged KV pool.

A step of ``LlamaForCausalLM`` (transformers models/llama/modeling_llama.py) runs
each layer as RMSNorm, q/k/v projections, rotary embedding, the KV write and paged
attention through the registered "paged|b200" function, o_proj, a residual add,
RMSNorm, gate/up projections, SiLU times up, down_proj and a residual add: about
twenty kernels per layer, most of them elementwise passes over the step's tokens.
``FusedLlamaStep`` runs the same step as nine launches per layer:

  add_rmsnorm (the previous residual add fused with this layer's input norm),
  one GEMM for q/k/v (the three weights concatenated once at set-up),
  rope_kv_append (rotary embedding of q and k fused with the K/V write to the pool),
  paged attention (decode rows on the split-K kernel, prefill rows on tcgen05),
  o_proj, add_rmsnorm, one GEMM for gate/up (concatenated), swiglu, down_proj,

then the final norm and lm_head on each row's last token only. Every kernel works
row by row, so one step may mix prefill chunks and decode rows. Rotary embedding
is bit-identical to HF's; RMSNorm and SiLU * up are computed in fp32 and rounded
once, where HF rounds an intermediate to the model's dtype first (at most one ulp
apart). bf16 / fp16 models only.
"""
from __future__ import annotations

import torch

from . import ops
from .paged_attention import paged_flash_attention


class FusedLlamaStep:
    """One step of `model` (prefill chunks and decode rows) with fused layer kernels."""

    def __init__(self, model):
        cfg = model.config
        dtype = next(model.parameters()).dtype
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"FusedLlamaStep: bf16 or fp16 model required, got {dtype}")
        inner = model.model
        self.hq = cfg.num_attention_heads
        self.hkv = cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.hidden = cfg.hidden_size
        self.eps = cfg.rms_norm_eps
        self.scale = self.head_dim ** -0.5
        self.dtype = dtype
        self.embed = inner.embed_tokens.weight
        self.final_norm = inner.norm.weight
        self.lm_head = model.lm_head.weight
        rot = inner.rotary_emb
        self.inv_freq = rot.inv_freq.float()
        self.rope_scaling = float(getattr(rot, "attention_scaling", 1.0))
        self.layers = []
        with torch.no_grad():
            for layer in inner.layers:
                at, mlp = layer.self_attn, layer.mlp
                lins = (at.q_proj, at.k_proj, at.v_proj, at.o_proj, mlp.gate_proj, mlp.up_proj, mlp.down_proj)
                if any(lin.bias is not None for lin in lins):
                    raise ValueError("FusedLlamaStep: projections with bias are not supported")
                if getattr(cfg, "hidden_act", "silu") != "silu":
                    raise ValueError(f"FusedLlamaStep: activation {cfg.hidden_act} is not supported (silu)")
                self.layers.append({
                    "wqkv": torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight]).contiguous(),
                    "wo": at.o_proj.weight,
                    "wgu": torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight]).contiguous(),
                    "wd": mlp.down_proj.weight,
                    "n1": layer.input_layernorm.weight,
                    "n2": layer.post_attention_layernorm.weight,
                })

    def rotary(self, positions: torch.Tensor):
        """cos, sin [rows, head_dim] as HF's rotary embedding computes them (fp32,
        then the model's dtype)."""
        freqs = positions.float()[:, None] * self.inv_freq[None, :]
        emb = torch.cat([freqs, freqs], dim=-1)
        return ((emb.cos() * self.rope_scaling).to(self.dtype), (emb.sin() * self.rope_scaling).to(self.dtype))

    @torch.inference_mode()
    def logits(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, kv_cache: torch.Tensor,
               metadata: dict, last: torch.Tensor | None = None) -> torch.Tensor:
        """tokens, positions, slots: [n_tokens] int64, the step's flattened tokens;
        kv_cache: [layers, 2, num_blocks, 16, kv heads, head_dim]; metadata: the
        step's paged metadata; last: the index of each row's last token (default:
        every token is a row's last, as in a decode step). Returns the logits of
        those tokens [rows, vocab]."""
        b = tokens.shape[0]
        cos, sin = self.rotary(positions)
        x = torch.index_select(self.embed, 0, tokens)  # residual stream, updated in place
        h = ops.add_rmsnorm(x, None, self.layers[0]["n1"], self.eps)
        for li, w in enumerate(self.layers):
            qkv = h @ w["wqkv"].t()
            kc, vc = kv_cache[li, 0], kv_cache[li, 1]
            q = ops.rope_kv_append(qkv, cos, sin, slots, kc, vc, self.hq, self.hkv)
            o, _ = paged_flash_attention(q, kc, vc, metadata, self.hq, self.hkv, self.scale)
            a = o.view(b, self.hq * self.head_dim) @ w["wo"].t()
            h = ops.add_rmsnorm(x, a, w["n2"], self.eps)
            dn = ops.swiglu(h @ w["wgu"].t()) @ w["wd"].t()
            nxt = self.layers[li + 1]["n1"] if li + 1 < len(self.layers) else self.final_norm
            h = ops.add_rmsnorm(x, dn, nxt, self.eps)
        if last is not None:
            h = h.index_select(0, last)
        return h @ self.lm_head.t()
