// pool.cu -- block mean pooling (one coalesced 128-bit HBM pass).
//
// Replaces block_mean_pool (attn_src/fft_attn/my_attn_v7.py:105-114) as used at
// :554-555.  The reference first materialises [L, H, D] copies of q and k
// (:528-530) and pools those; this kernel reads [B, H, L, D] in place with any
// (b, h, l) strides, so the copies disappear.
//
// One CTA of 256 threads pools one (b, h, block).  With G = D / VEC 16-byte
// lanes (VEC = 8 bf16 or 4 fp32 channels) and P = 256 / G row phases, thread
// (p, g) sums rows p, p+P, ... of channels [g*VEC, g*VEC+VEC) in fp32 in row
// order (padded rows contribute +0), the P partials are combined by the tree
// part[p] += part[p+s] for s = P/2 .. 1, and the total is divided by
// block_size and rounded to the input dtype.  This order is the canonical one
// the CPU oracle restates.  A warp reads two or four whole rows per 16-byte
// load instruction, so every access is a fully used 512-byte transaction.

#include "ffts_common.cuh"

namespace ffts {

template <typename T>
__global__ void __launch_bounds__(256) pool_kernel(const T *__restrict__ x, int64_t H, int64_t L,
                                                   int D, int64_t sb, int64_t sh, int64_t sl,
                                                   int bs, int64_t N, T *__restrict__ out) {
  constexpr int VEC = Elem<T>::kVec;
  extern __shared__ float part[];  // [P][D]
  const int G = D / VEC;
  const int P = 256 / G;
  const int tid = threadIdx.x;
  const int g = tid % G;
  const int p = tid / G;
  const int64_t n = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / H, h = bh % H;
  const T *base = x + b * sb + h * sh + int64_t(g) * VEC;

  float acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;

  // Rows in groups of 8 so that eight independent 16-byte loads are in flight.
  for (int r0 = p; r0 < bs; r0 += 8 * P) {
    float v[8][VEC];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = r0 + u * P;
      const int64_t t = n * bs + r;
      if (r < bs && t < L) {
        load_vec_f32<T>(base + t * sl, v[u]);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[u][e] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (r0 + u * P < bs) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = __fadd_rn(acc[e], v[u][e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) part[p * D + g * VEC + e] = acc[e];
  __syncthreads();
  for (int s = P / 2; s >= 1; s >>= 1) {
    if (p < s) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int i = g * VEC + e;
        part[p * D + i] = __fadd_rn(part[p * D + i], part[(p + s) * D + i]);
      }
    }
    __syncthreads();
  }
  if (p == 0) {
    T res[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      res[e] = Elem<T>::from_f32(__fdiv_rn(part[g * VEC + e], (float)bs));
    T *o = out + (bh * N + n) * D + g * VEC;
    *reinterpret_cast<uint4 *>(o) = *reinterpret_cast<const uint4 *>(res);
  }
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
  const int G = int(D / vec), P = 256 / G;
  const size_t smem = size_t(P) * D * sizeof(float);
  dim3 grid(unsigned(N), unsigned(B * H));
  if (dtype == FFTS_DTYPE_BF16)
    pool_kernel<__nv_bfloat16><<<grid, 256, smem, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), H, L, int(D), sb, sh, sl, bs, N,
        static_cast<__nv_bfloat16 *>(out));
  else
    pool_kernel<float><<<grid, 256, smem, stream>>>(static_cast<const float *>(x), H, L, int(D), sb,
                                                    sh, sl, bs, N, static_cast<float *>(out));
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
