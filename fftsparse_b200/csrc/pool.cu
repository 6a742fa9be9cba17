// pool.cu -- block mean pooling (one coalesced 128-bit HBM pass).
//
// Replaces block_mean_pool (attn_src/fft_attn/my_attn_v7.py:105-114) as used at
// :554-555.  The reference first materialises [L, H, D] copies of q and k
// (:528-530) and pools those; this kernel reads [B, H, L, D] in place with any
// (b, h, l) strides, so the copies disappear.
//
// A CTA of 256 threads pools 256/G blocks of one (b, h), where G = D / VEC
// 16-byte lanes span a row (VEC = 8 bf16 or 4 fp32 channels).  Thread (s, g)
// sums rows 0 .. block_size-1 of block s in its VEC channels in fp32, in row
// order (rows past L contribute +0), then divides by block_size and rounds to
// the input dtype: the canonical order the CPU oracle restates.  No shared
// memory and no barriers; sixteen 16-byte loads per thread are in flight at a
// time, and a warp's load instruction reads whole 256-byte rows.

#include "ffts_common.cuh"

namespace ffts {

template <typename T>
__global__ void __launch_bounds__(256) pool_kernel(const T *__restrict__ x, int64_t H, int64_t L,
                                                   int D, int64_t sb, int64_t sh, int64_t sl,
                                                   int bs, int64_t N, T *__restrict__ out) {
  constexpr int VEC = Elem<T>::kVec;
  constexpr int U = 16;  // loads in flight per thread
  const int G = D / VEC;
  const int per_cta = 256 / G;
  const int g = threadIdx.x % G;
  const int64_t n = int64_t(blockIdx.x) * per_cta + threadIdx.x / G;
  const int64_t bh = blockIdx.y;
  if (n >= N) return;
  const int64_t b = bh / H, h = bh % H;
  const T *base = x + b * sb + h * sh + int64_t(g) * VEC;
  float acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;
  for (int r0 = 0; r0 < bs; r0 += U) {
    uint4 raw[U];  // the 16-byte words of U rows, widened during the in-order adds
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t t = n * bs + r0 + u;
      raw[u] = (r0 + u < bs && t < L) ? *reinterpret_cast<const uint4 *>(base + t * sl) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (r0 + u < bs) {
        float v[VEC];
        widen_vec<T>(raw[u], v);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = __fadd_rn(acc[e], v[e]);
      }
    }
  }
  T res[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) res[e] = Elem<T>::from_f32(__fdiv_rn(acc[e], (float)bs));
  T *o = out + (bh * N + n) * D + g * VEC;
  *reinterpret_cast<uint4 *>(o) = *reinterpret_cast<const uint4 *>(res);
}

int launch_pool(const void *x, int dtype, int64_t B, int64_t H, int64_t L, int64_t D,
                int64_t sb, int64_t sh, int64_t sl, int bs, void *out, cudaStream_t stream) {
  const int vec = dtype == FFTS_DTYPE_BF16 ? 8 : 4;
  FFTS_REQUIRE(dtype == FFTS_DTYPE_BF16 || dtype == FFTS_DTYPE_F32, "pool: unsupported dtype %d", dtype);
  FFTS_REQUIRE(B > 0 && H > 0 && L > 0 && D > 0 && bs > 0, "pool: empty or negative shape");
  FFTS_REQUIRE(D % vec == 0 && 256 % (D / vec) == 0,
               "pool: head_dim %lld must be a power-of-two multiple of %d up to %d", (long long)D,
               vec, 256 * vec);
  FFTS_REQUIRE(sb % vec == 0 && sh % vec == 0 && sl % vec == 0,
               "pool: strides must be multiples of 16 bytes");
  FFTS_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0,
               "pool: pointers must be 16-byte aligned");
  FFTS_REQUIRE(B * H <= 65535, "pool: B*H too large");
  const int64_t N = ceil_div(L, bs);
  const int G = int(D / vec), per_cta = 256 / G;
  dim3 grid(unsigned(ceil_div(N, per_cta)), unsigned(B * H));
  if (dtype == FFTS_DTYPE_BF16)
    pool_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), H, L, int(D), sb, sh, sl, bs, N,
        static_cast<__nv_bfloat16 *>(out));
  else
    pool_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float *>(x), H, L, int(D), sb,
                                                    sh, sl, bs, N, static_cast<float *>(out));
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
