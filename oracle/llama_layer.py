"""Unquantised Llama decoder layer in plain torch with autograd (TEST INFRASTRUCTURE ONLY): what the
COAT layer (coat/models/coat_llama.py:1084-1181) approximates in FP8.  RMSNorm (eps 1e-5, the value
hard-coded in the reference's autograd blocks, coat_llama.py:246,626), q/k/v projections, default RoPE,
causal attention, o projection, residual, RMSNorm, SiLU-gated MLP, residual.

Parity unpinned: the reference's own layer test (tests/test_coat_llamalayer.py) is bit-rotted and needs a
checkpoint from the network, so the FP8 layer is checked against this layer at FP8-level tolerances
stated in the test, not against reference outputs."""
import torch
import torch.nn.functional as F


def _rope(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


def reference_layer(x, w, n_heads, n_kv_heads, rope_theta=10000.0, eps=1e-5):
    """x [B,S,H]; w: dict with q,k,v,o,gate,up,down ([out,in]) and ln1, ln2 ([H]).  Computation in x.dtype
    (use fp32 or fp64 tensors for the checker)."""
    B, S, H = x.shape
    hd = H // n_heads

    def rms(t, g):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * g

    h = rms(x, w["ln1"])
    q = (h @ w["q"].t()).view(B, S, n_heads, hd).transpose(1, 2)
    k = (h @ w["k"].t()).view(B, S, n_kv_heads, hd).transpose(1, 2)
    v = (h @ w["v"].t()).view(B, S, n_kv_heads, hd).transpose(1, 2)
    pos = torch.arange(S, device=x.device, dtype=torch.float32)
    inv = 1.0 / (rope_theta ** (torch.arange(0, hd, 2, device=x.device, dtype=torch.float32) / hd))
    emb = torch.cat((pos[:, None] * inv, pos[:, None] * inv), dim=-1)
    cos, sin = emb.cos().to(x.dtype), emb.sin().to(x.dtype)
    q, k = _rope(q, cos, sin), _rope(k, cos, sin)
    if n_kv_heads != n_heads:
        k = k.repeat_interleave(n_heads // n_kv_heads, dim=1)
        v = v.repeat_interleave(n_heads // n_kv_heads, dim=1)
    a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, S, H)
    x = x + a @ w["o"].t()
    h = rms(x, w["ln2"])
    return x + (F.silu(h @ w["gate"].t()) * (h @ w["up"].t())) @ w["down"].t()
