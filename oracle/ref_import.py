"""Run the reference's own ``myattn_prefill`` mask path on the CPU.

TEST INFRASTRUCTURE, used only to generate and check golden fixtures in a
container that holds the reference checkout (it is never present where the
GPU tests or the bench run; nothing on the product path imports this file).

The reference module attn_src/fft_attn/my_attn_v7.py is imported unmodified.
Three things stand in for what this container lacks:

* ``matplotlib`` (imported by attn_src/fft_attn/vis_utils.py:4-5) is stubbed,
  since the visualisation paths are off at every call site;
* ``block_sparse_attn`` (imported at my_attn_v7.py:7, a third-party CUDA wheel
  that is neither vendored nor installed) is replaced by a function that
  records ``base_blockmask`` and returns a CPU restatement of its attention;
* the ``assert query_states.is_cuda`` at my_attn_v7.py:502 is satisfied by a
  tensor subclass whose ``is_cuda`` property answers True; every tensor op
  still runs on the CPU.

Optional canonicalisation (``stable_topk=True``): ``torch.topk`` inside the
reference module is replaced by a stable descending sort + slice, so ties are
broken by lowest index (torch.topk leaves tie order unspecified).  This is the
tie rule the build's kernels implement.
"""
from __future__ import annotations

import importlib
import os
import sys
import types

import torch

# The reference checkout is named explicitly by the caller; there is no default path.
REF_ROOT = os.environ.get("FFTS_REFERENCE_ROOT", "")

_captured: dict = {}
_module = None


class _CudaClaim(torch.Tensor):
    """CPU tensor that reports ``is_cuda`` so the reference's device assert passes."""

    @property
    def is_cuda(self):  # type: ignore[override]
        return True


def _stub_matplotlib():
    if "matplotlib" in sys.modules:
        return
    mpl = types.ModuleType("matplotlib")
    plt = types.ModuleType("matplotlib.pyplot")
    patches = types.ModuleType("matplotlib.patches")
    mpl.pyplot = plt
    mpl.patches = patches
    mpl.use = lambda *a, **k: None
    sys.modules["matplotlib"] = mpl
    sys.modules["matplotlib.pyplot"] = plt
    sys.modules["matplotlib.patches"] = patches


def cpu_block_sparse_attention(q_unpad, k_unpad, v_unpad, mask, block_size, causal=True):
    """fp32 CPU restatement of block_sparse_attn_func's forward semantics.

    q/k/v are [L, H, D]; mask is bool [1, H, Nq, Nk]; query row t in q-block i
    attends to keys s (s <= t when causal) whose k-block j has mask[0, h, i, j];
    scale 1/sqrt(D); rows with nothing selected produce zeros.
    """
    L, H, D = q_unpad.shape
    out = torch.zeros(L, H, D, dtype=torch.float32)
    scale = 1.0 / (D ** 0.5)
    m = mask[0].to(torch.bool)
    tok_blk = torch.arange(L) // block_size
    for h in range(H):
        qh = q_unpad[:, h].float()
        kh = k_unpad[:, h].float()
        vh = v_unpad[:, h].float()
        for i in range(m.shape[1]):
            r0, r1 = i * block_size, min(L, (i + 1) * block_size)
            if r0 >= L:
                break
            sel = m[i][tok_blk]  # [L] keys whose block is selected
            if causal:
                allowed = sel[None, :] & (torch.arange(L)[None, :] <= torch.arange(r0, r1)[:, None])
            else:
                allowed = sel[None, :].expand(r1 - r0, L)
            s = (qh[r0:r1] @ kh.T) * scale
            s = s.masked_fill(~allowed, float("-inf"))
            any_row = allowed.any(dim=1, keepdim=True)
            p = torch.softmax(s.masked_fill(~any_row, 0.0), dim=-1) * any_row
            out[r0:r1, h] = p @ vh
    return out


def _block_sparse_attn_stub(q_unpad, k_unpad, v_unpad, cu_q, cu_k, head_mask_type=None,
                            streaming_info=None, base_blockmask=None, max_seqlen_q_=None,
                            max_seqlen_k_=None, p_dropout=0.0, deterministic=True,
                            is_causal=True, **_):
    _captured["mask"] = base_blockmask.detach().clone().as_subclass(torch.Tensor)
    if _captured.get("skip_attention", True):
        return torch.zeros_like(q_unpad.as_subclass(torch.Tensor))
    bs = _captured["block_size"]
    out = cpu_block_sparse_attention(q_unpad.as_subclass(torch.Tensor),
                                     k_unpad.as_subclass(torch.Tensor),
                                     v_unpad.as_subclass(torch.Tensor),
                                     _captured["mask"], bs, is_causal)
    return out.to(q_unpad.dtype)


def _flash_attn_stub(q, k, v, causal=True, **_):
    """Dense causal attention on [B, L, H, D] (the short-sequence branch)."""
    q, k, v = (t.as_subclass(torch.Tensor).float() for t in (q, k, v))
    B, L, H, D = q.shape
    s = torch.einsum("blhd,bshd->bhls", q, k) / (D ** 0.5)
    if causal:
        s = s.masked_fill(torch.ones(L, L, dtype=torch.bool).triu(1), float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhls,bshd->blhd", p, v)


def load_reference():
    """Import attn_src.fft_attn.my_attn_v7 from the reference checkout (CPU stubs)."""
    global _module
    if _module is not None:
        return _module
    if not REF_ROOT:
        raise RuntimeError("set FFTS_REFERENCE_ROOT to the root of a PureEidolon/FFTSparse checkout")
    if not os.path.isdir(os.path.join(REF_ROOT, "attn_src")):
        raise RuntimeError(f"reference checkout not found at FFTS_REFERENCE_ROOT={REF_ROOT}")
    _stub_matplotlib()
    bsa = types.ModuleType("block_sparse_attn")
    bsa.block_sparse_attn_func = _block_sparse_attn_stub
    sys.modules["block_sparse_attn"] = bsa
    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    mod = importlib.import_module("attn_src.fft_attn.my_attn_v7")
    mod.block_sparse_attn_func = _block_sparse_attn_stub
    mod.flash_attn_func = _flash_attn_stub
    _module = mod
    return mod


class _StableTorch:
    """Proxy for the ``torch`` module with a tie-stable ``topk``."""

    def __init__(self, real):
        self._real = real

    def __getattr__(self, name):
        return getattr(self._real, name)

    def topk(self, input, k, dim=-1, largest=True, sorted=True):
        vals, idx = self._real.sort(input, dim=dim, descending=largest, stable=True)
        return vals.narrow(dim, 0, k), idx.narrow(dim, 0, k)


def run_reference(q, k, v, *, layer_idx=0, stable_topk=True, with_attention=False, **kwargs):
    """Call the reference ``myattn_prefill`` on CPU tensors [1, H, L, D].

    Returns ``(mask, out)``: the boolean block mask handed to the attention
    kernel (``base_blockmask``, [1, H, Nq, Nk]) and the operator's output
    ([1, L, H*D], zeros unless ``with_attention``).
    """
    mod = load_reference()
    _captured.clear()
    _captured["skip_attention"] = not with_attention
    _captured["block_size"] = kwargs.get("block_size", 128)
    real_torch = mod.torch
    if stable_topk:
        mod.torch = _StableTorch(real_torch)
    try:
        with torch.no_grad():
            out = mod.myattn_prefill(q.as_subclass(_CudaClaim), k.as_subclass(_CudaClaim),
                                     v.as_subclass(_CudaClaim), layer_idx, **kwargs)
    finally:
        mod.torch = real_torch
    return _captured.get("mask"), out.as_subclass(torch.Tensor)


def reference_intermediates(q, k, *, block_size=128, sink_ratio=0.1, recent_ratio=0.1,
                            local_span_ratio=0.1, stable_topk=True):
    """Pooled blocks and FFT correlation scores computed by the reference's functions."""
    mod = load_reference()
    H, L = q.shape[1], q.shape[2]
    N = (L + block_size - 1) // block_size
    keep_sink = max(1, int(N * sink_ratio))
    local_window = max(2, int(N * local_span_ratio)) // 2
    q_unpad = q.squeeze(0).transpose(0, 1).contiguous()
    k_unpad = k.squeeze(0).transpose(0, 1).contiguous()
    Qb = mod.block_mean_pool(q_unpad, block_size)
    Kb = mod.block_mean_pool(k_unpad, block_size)
    corr, corr_sum, _, _ = mod.batch_fft_cross_correlation(Qb, Kb, local_window=local_window,
                                                           keep_sink=keep_sink)
    return {"Qb": Qb, "Kb": Kb, "corr": corr, "corr_sum": corr_sum}
