// rope_pool.cu -- the caller's rotary embedding, the head-major layout and the
// block pooling of q and k in one HBM pass.
//
// The caller of myattn_prefill (eval/LongBench/pred.py:177-194) projects q, k
// and v token-major, views them head-major, applies HF apply_rotary_pos_emb
// (x * cos + rotate_half(x) * sin, in bf16), and myattn_prefill then pools the
// rotated q and k (block_mean_pool, attn_src/fft_attn/my_attn_v7.py:105-114,
// used at :554-555).  Evaluated by torch that is a handful of elementwise passes
// over q and k plus the pooling pass.  This kernel reads each projection row
// once and writes the rotated head-major q and k, the head-major v, and the
// pooled q and k blocks.
//
// Arithmetic (bit-identical to the torch expression, then to pool_kernel): per
// element a = bf16(x * cos), b = bf16(r * sin) with r = -x[d + D/2] (d < D/2) or
// x[d - D/2], out = bf16(a + b), every operation in fp32 with round-to-nearest
// (evaluated as packed bf16 multiplies and adds, which round the same way);
// the pooled value of a channel is the fp32 sum of the block's rotated bf16
// values in row order from +0, divided by block_size and rounded to bf16.
//
// A thread owns one pool block and 8 channels of each half of the head (the
// RoPE partners d and d + D/2 sit in the same thread), walking the block's rows
// in order with 2 rows of loads in flight; 8 threads cover a row, a warp 4
// blocks, so every load and store instruction moves whole 128-byte segments.

#include "ffts_common.cuh"

namespace ffts {
namespace rope {

constexpr int kD = 128;        // head_dim
constexpr int kHalf = kD / 2;  // RoPE pairs (d, d + 64)
constexpr int kThreadsPerBlk = kHalf / 8;
constexpr int kBlocksPerCta = 256 / kThreadsPerBlk;
constexpr int kU = 2;          // rows of loads in flight per thread (2 CTAs per SM: 96 KB in flight)

struct Args {
  const __nv_bfloat16 *src[3];  // q, k, v projections (token-major); src[2] may be NULL
  int64_t ld[3];                // their row strides (elements)
  __nv_bfloat16 *dst[3];        // head-major [heads, L, D] outputs
  __nv_bfloat16 *pooled[2];     // [heads, N, D] block means of the rotated q and k
  const __nv_bfloat16 *cos, *sin;
  int64_t cs_ld;
  int64_t L, N;
  int Hq, Hkv, bs;
};

__device__ __forceinline__ void unpack8(const uint4 &w, float *f) {
  const __nv_bfloat162 *p = reinterpret_cast<const __nv_bfloat162 *>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(p[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float *f) {
  uint4 w;
  uint32_t *u = reinterpret_cast<uint32_t *>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat162 pr = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
    u[e] = *reinterpret_cast<const uint32_t *>(&pr);
  }
  return w;
}

__global__ void __launch_bounds__(256, 2) rope_pool_kernel(const __grid_constant__ Args a) {
  const int g = threadIdx.x % kThreadsPerBlk;  // channels [8g, 8g+8) and [64+8g, 64+8g+8)
  const int64_t n = int64_t(blockIdx.x) * kBlocksPerCta + threadIdx.x / kThreadsPerBlk;
  if (n >= a.N) return;
  int head = blockIdx.y, role = 0;
  if (head >= a.Hq) {
    head -= a.Hq;
    role = 1;
    if (head >= a.Hkv) {
      head -= a.Hkv;
      role = 2;
    }
  }
  const __nv_bfloat16 *src = a.src[role] + int64_t(head) * kD + 8 * g;
  const int64_t ld = a.ld[role];
  __nv_bfloat16 *dst = a.dst[role] + int64_t(head) * a.L * kD + 8 * g;
  const int64_t t0 = n * a.bs;
  const int rows = a.L - t0 < int64_t(a.bs) ? int(a.L - t0) : a.bs;

  if (role == 2) {  // v: layout only
    for (int r0 = 0; r0 < rows; r0 += kU) {
      uint4 lo[kU], hi[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (r0 + u < rows && FFTS_IN_RANGE(t0 + r0 + u, a.L)) {
          const __nv_bfloat16 *p = src + (t0 + r0 + u) * ld;
          lo[u] = *reinterpret_cast<const uint4 *>(p);
          hi[u] = *reinterpret_cast<const uint4 *>(p + kHalf);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (r0 + u < rows && FFTS_IN_RANGE(t0 + r0 + u, a.L)) {
          __nv_bfloat16 *p = dst + (t0 + r0 + u) * kD;
          *reinterpret_cast<uint4 *>(p) = lo[u];
          *reinterpret_cast<uint4 *>(p + kHalf) = hi[u];
        }
      }
    }
    return;
  }

  const __nv_bfloat16 *cs = a.cos + 8 * g, *sn = a.sin + 8 * g;
  float acc_lo[8], acc_hi[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc_lo[e] = acc_hi[e] = 0.0f;
  for (int r0 = 0; r0 < rows; r0 += kU) {
    uint4 xl[kU], xh[kU], cl[kU], ch[kU], sl[kU], sh[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (r0 + u < rows && FFTS_IN_RANGE(t0 + r0 + u, a.L)) {
        const int64_t t = t0 + r0 + u;
        const __nv_bfloat16 *p = src + t * ld;
        xl[u] = *reinterpret_cast<const uint4 *>(p);
        xh[u] = *reinterpret_cast<const uint4 *>(p + kHalf);
        cl[u] = *reinterpret_cast<const uint4 *>(cs + t * a.cs_ld);
        ch[u] = *reinterpret_cast<const uint4 *>(cs + t * a.cs_ld + kHalf);
        sl[u] = *reinterpret_cast<const uint4 *>(sn + t * a.cs_ld);
        sh[u] = *reinterpret_cast<const uint4 *>(sn + t * a.cs_ld + kHalf);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (r0 + u < rows && FFTS_IN_RANGE(t0 + r0 + u, a.L)) {
        // packed bf16 arithmetic: a bf16 x bf16 product is exact in fp32, so
        // mul.rn.bf16x2 rounds it once exactly as bf(x * c) does; the sum of two
        // bf16 values rounds in add.rn.bf16x2 as bf(a + b) does (exact in fp32
        // when their exponents are within 16, else the larger value is the result
        // both ways)
        const uint32_t xa[4] = {xl[u].x, xl[u].y, xl[u].z, xl[u].w}, xb[4] = {xh[u].x, xh[u].y, xh[u].z, xh[u].w};
        const uint32_t ca[4] = {cl[u].x, cl[u].y, cl[u].z, cl[u].w}, cb[4] = {ch[u].x, ch[u].y, ch[u].z, ch[u].w};
        const uint32_t sa[4] = {sl[u].x, sl[u].y, sl[u].z, sl[u].w}, sb[4] = {sh[u].x, sh[u].y, sh[u].z, sh[u].w};
        uint32_t o1[4], o2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o1[e] = bf16x2_add(bf16x2_mul(xa[e], ca[e]), bf16x2_mul(bf16x2_neg(xb[e]), sa[e]));
          o2[e] = bf16x2_add(bf16x2_mul(xb[e], cb[e]), bf16x2_mul(xa[e], sb[e]));
          acc_lo[2 * e] = __fadd_rn(acc_lo[2 * e], __uint_as_float(o1[e] << 16));
          acc_lo[2 * e + 1] = __fadd_rn(acc_lo[2 * e + 1], __uint_as_float(o1[e] & 0xffff0000u));
          acc_hi[2 * e] = __fadd_rn(acc_hi[2 * e], __uint_as_float(o2[e] << 16));
          acc_hi[2 * e + 1] = __fadd_rn(acc_hi[2 * e + 1], __uint_as_float(o2[e] & 0xffff0000u));
        }
        const uint4 w1 = make_uint4(o1[0], o1[1], o1[2], o1[3]), w2 = make_uint4(o2[0], o2[1], o2[2], o2[3]);
        __nv_bfloat16 *p = dst + (t0 + r0 + u) * kD;
        *reinterpret_cast<uint4 *>(p) = w1;
        *reinterpret_cast<uint4 *>(p + kHalf) = w2;
      }
    }
  }
  // rows past L contribute +0, which leaves a sum that started at +0 unchanged
  const float inv_n = float(a.bs);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    acc_lo[e] = __fdiv_rn(acc_lo[e], inv_n);
    acc_hi[e] = __fdiv_rn(acc_hi[e], inv_n);
  }
  __nv_bfloat16 *po = a.pooled[role] + (int64_t(head) * a.N + n) * kD + 8 * g;
  *reinterpret_cast<uint4 *>(po) = pack8(acc_lo);
  *reinterpret_cast<uint4 *>(po + kHalf) = pack8(acc_hi);
}

}  // namespace rope

int launch_rope_pool(const void *q_src, int64_t q_ld, const void *k_src, int64_t k_ld, const void *v_src,
                     int64_t v_ld, int64_t L, int64_t Hq, int64_t Hkv, int64_t D, const void *cos, const void *sin,
                     int64_t cs_ld, int bs, void *q_out, void *k_out, void *v_out, void *q_pooled, void *k_pooled,
                     cudaStream_t stream) {
  using namespace rope;
  FFTS_REQUIRE(q_src && k_src && cos && sin && q_out && k_out && q_pooled && k_pooled && (!v_src || v_out),
               "rope_pool: NULL argument");
  FFTS_REQUIRE(D == kD, "rope_pool: head_dim must be %d (got %lld)", kD, (long long)D);
  FFTS_REQUIRE(L >= 1 && Hq >= 1 && Hkv >= 1 && bs >= 1, "rope_pool: empty or negative shape");
  FFTS_REQUIRE(Hq + 2 * Hkv <= 65535, "rope_pool: too many heads");
  FFTS_REQUIRE(q_ld >= Hq * D && k_ld >= Hkv * D && (!v_src || v_ld >= Hkv * D) && cs_ld >= D,
               "rope_pool: a row stride is shorter than its row");
  FFTS_REQUIRE(q_ld % 8 == 0 && k_ld % 8 == 0 && v_ld % 8 == 0 && cs_ld % 8 == 0,
               "rope_pool: row strides must be multiples of 16 bytes");
  for (const void *p : {q_src, k_src, v_src, cos, sin, (const void *)q_out, (const void *)k_out,
                        (const void *)v_out, (const void *)q_pooled, (const void *)k_pooled})
    FFTS_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15) == 0, "rope_pool: pointers must be 16-byte aligned");
  Args a{};
  a.src[0] = static_cast<const __nv_bfloat16 *>(q_src);
  a.src[1] = static_cast<const __nv_bfloat16 *>(k_src);
  a.src[2] = static_cast<const __nv_bfloat16 *>(v_src);
  a.ld[0] = q_ld;
  a.ld[1] = k_ld;
  a.ld[2] = v_ld;
  a.dst[0] = static_cast<__nv_bfloat16 *>(q_out);
  a.dst[1] = static_cast<__nv_bfloat16 *>(k_out);
  a.dst[2] = static_cast<__nv_bfloat16 *>(v_out);
  a.pooled[0] = static_cast<__nv_bfloat16 *>(q_pooled);
  a.pooled[1] = static_cast<__nv_bfloat16 *>(k_pooled);
  a.cos = static_cast<const __nv_bfloat16 *>(cos);
  a.sin = static_cast<const __nv_bfloat16 *>(sin);
  a.cs_ld = cs_ld;
  a.L = L;
  a.N = ceil_div(L, bs);
  a.Hq = int(Hq);
  a.Hkv = int(Hkv);
  a.bs = bs;
  const int heads = int(Hq + Hkv + (v_src ? Hkv : 0));
  dim3 grid(unsigned(ceil_div(a.N, kBlocksPerCta)), unsigned(heads));
  rope_pool_kernel<<<grid, 256, 0, stream>>>(a);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
