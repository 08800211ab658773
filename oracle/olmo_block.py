"""Unquantised OLMo sequential block in plain torch with autograd (TEST INFRASTRUCTURE ONLY): what the COAT block
(coat/models/coat_olmo.py:910-1076) approximates in FP8, in the OLMo-7B configuration: LayerNorm without
parameters (eps 1e-5), one fused q/k/v projection, rotary embedding, causal attention, output projection,
residual, LayerNorm, `ff_proj` whose output halves are (up, gate) in that order, silu(gate) * up, `ff_out`,
residual (the unquantised branches of the same file, :1019-1070, with olmo/model.py's SwiGLU: `x, gate =
x.chunk(2, dim=-1); silu(gate) * x`).

Parity unpinned: the reference's block needs the host trainer's package and its yaml configuration to be
constructed, so the FP8 block is checked against this block at FP8-level tolerances stated in the test, and against
the same composition on the reference's operators."""
import torch
import torch.nn.functional as F

from .llama_layer import _rope


def reference_block(x, w, n_heads, n_kv_heads=None, rope_theta=10000.0, eps=1e-5):
    """x [B,T,D]; w: dict with att_proj [D + 2*kv, D], attn_out [D, D], ff_proj [2I, D], ff_out [D, I].
    Computation in x.dtype (use fp32 or fp64 tensors for the checker)."""
    B, T, D = x.shape
    n_kv_heads = n_kv_heads or n_heads
    hd = D // n_heads

    def ln(t):
        return F.layer_norm(t, (D,), None, None, eps)

    qkv = ln(x) @ w["att_proj"].t()
    q, k, v = qkv.split((D, n_kv_heads * hd, n_kv_heads * hd), dim=-1)
    q = q.reshape(B, T, n_heads, hd).transpose(1, 2)
    k = k.reshape(B, T, n_kv_heads, hd).transpose(1, 2)
    v = v.reshape(B, T, n_kv_heads, hd).transpose(1, 2)
    pos = torch.arange(T, device=x.device, dtype=torch.float32)
    inv = 1.0 / (rope_theta ** (torch.arange(0, hd, 2, device=x.device, dtype=torch.float32) / hd))
    emb = torch.cat((pos[:, None] * inv, pos[:, None] * inv), dim=-1)
    cos, sin = emb.cos().to(x.dtype), emb.sin().to(x.dtype)
    q, k = _rope(q, cos, sin), _rope(k, cos, sin)
    if n_kv_heads != n_heads:
        k = k.repeat_interleave(n_heads // n_kv_heads, dim=1)
        v = v.repeat_interleave(n_heads // n_kv_heads, dim=1)
    a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, T, D)
    x = x + a @ w["attn_out"].t()
    up, gate = (ln(x) @ w["ff_proj"].t()).chunk(2, dim=-1)
    return x + (F.silu(gate) * up) @ w["ff_out"].t()
