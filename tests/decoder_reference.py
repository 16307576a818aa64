"""Independent restatement of one Llama decode step, for the decoder tests.

Not a test module (pytest collects only test_*.py). Written per head with
plain torch ops in fp32 from a decoder's own weights and caches; nothing of
the decoder's step, fused kernels or tensor-parallel split is used. With
``storage=torch.float16`` every activation the decoder keeps in fp16 (the
residual stream after each add, normalised inputs, linear outputs, rotated
heads, attention outputs, SwiGLU output) is rounded to fp16 at the same
points, so that what remains between the two is the kernels' arithmetic
(fp32 accumulation order, fused steps) and not the model's storage format.
"""

from __future__ import annotations

import math

import torch

from dequant_project_b200.packer import dequantize


def reference_step(dec, tokens, pos, storage=None):
    """Logits [M, vocab] fp32 of a world-1 ``TPDecoder`` at position ``pos``
    (call before the decoder's own step writes cache slot ``pos``)."""
    cfg, d = dec.cfg, dec.cfg.head_dim
    if dec.world != 1:
        raise ValueError("the restatement reads a world-1 decoder's full weights")
    rnd = (lambda t: t.to(storage).float()) if storage is not None else (lambda t: t)
    m = tokens.shape[0]
    h = dec.embed[tokens].float()
    dev = h.device
    inv = cfg.rope_theta ** (-torch.arange(0, d, 2, dtype=torch.float64, device=dev) / d)
    ang = pos * inv
    cos = torch.cat([ang.cos(), ang.cos()]).float()
    sin = torch.cat([ang.sin(), ang.sin()]).float()

    def norm(x):
        return rnd(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.eps))

    def rope(t):
        half = d // 2
        return rnd(t * cos + torch.cat([-t[..., half:], t[..., :half]], dim=-1) * sin)

    def linear(x, pw):
        return rnd(x @ dequantize(pw).float().t())

    nq, nkv = cfg.n_heads * d, cfg.n_kv_heads * d
    group = cfg.n_heads // cfg.n_kv_heads
    for layer, w in enumerate(dec.layers):
        qkv = linear(norm(h), w["qkv"])
        q = rope(qkv[:, :nq].reshape(m, cfg.n_heads, d))
        k = rope(qkv[:, nq:nq + nkv].reshape(m, cfg.n_kv_heads, d))
        v = qkv[:, nq + nkv:].reshape(m, cfg.n_kv_heads, d)
        kc = dec.k_cache[layer][:, :, :pos].float()
        vc = dec.v_cache[layer][:, :, :pos].float()
        out = torch.empty(m, cfg.n_heads, d, device=dev)
        for b in range(m):
            for hh in range(cfg.n_heads):
                kv = hh // group
                keys = torch.cat([kc[b, kv], k[b, kv][None]])
                vals = torch.cat([vc[b, kv], v[b, kv][None]])
                p = torch.softmax(keys @ q[b, hh] / math.sqrt(d), dim=0)
                out[b, hh] = p @ vals
        h = rnd(h + linear(rnd(out).reshape(m, nq), w["o"]))
        gu = linear(norm(h), w["gu"])
        if getattr(dec, "gu_order", None) is not None:   # rows stored interleaved by eights
            gu = gu[:, torch.argsort(dec.gu_order.to(gu.device))]
        i = gu.shape[1] // 2
        act = rnd(torch.nn.functional.silu(gu[:, :i]) * gu[:, i:])
        h = rnd(h + linear(act, w["down"]))
    head = dec.lm_head
    x = norm(h)
    return x @ (dequantize(head).float() if hasattr(head, "qweight") else head.float()).t()


def max_rel_err(a, b) -> float:
    """max|a - b| / max|b| over all elements (fp32)."""
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max()).item()
