"""fftsparse_b200: the FFTSparse prefill hot path, B200-native (sm_100a).

Public surface (mirrors attn_src/fft_attn/my_attn_v7.py):

  myattn_prefill(q, k, v, layer_idx, ...)   drop-in for the reference operator
  myattn_prefill_host(q, k, v, layer_idx)   the same on pinned host buffers, copies overlapped per head chunk
  fft_block_mask(q, k, ...)                 the selected block mask + statistics
  sparse_attention(q, k, v, bits, bs)       block-sparse attention on packed bits
  pool_blocks(x, bs)                        block mean pooling
  rope_pool(q_proj, k_proj, v_proj, ...)    the caller's RoPE + head-major layout + pooling, one pass
  qkv_rope_pool(hidden, weight, bias, ...)  the QKV projection GEMM with all of rope_pool in its epilogue
  derive_mask_params(L, ...)                host-side parameter derivation
  calibrate.calibrate_from_qk(layers, t)    target-sparsity calibration on the device
  decode_attention(q, k_cache, v_cache)     one-token decode over the un-expanded KV cache
  dist.sharded_prefill(...)                 KV-group sharded prefill (peer-memory all-gather)
  check_status(device=None)                 raise WaitTimeout if a kernel's bounded wait ran out
"""
from .params import derive_mask_params, MaskParams  # noqa: F401
from .prefill import (  # noqa: F401
    AttentionCache,
    BlockMask,
    _attention_cache,
    fft_block_mask,
    myattn_prefill,
    myattn_prefill_host,
    pool_blocks,
    qkv_rope_pool,
    rope_pool,
    sparse_attention,
)
from .decode import decode_attention  # noqa: F401
from .status import WaitTimeout, check_status  # noqa: F401
from ._lib import load as load_library, LIB_PATH  # noqa: F401

__version__ = "0.1.0"
