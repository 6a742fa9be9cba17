// decode.cu -- single-token decode attention over a head-major KV cache.
//
// Replaces the caller's eager decode branch (eval/LongBench/pred.py:306-322:
// softmax(q k^T / sqrt(D)) v over the whole cache with repeat_kv-expanded k/v,
// fp32 softmax).  It reads the cache un-expanded, [B, Hkv, Lk, D] bf16 (the
// layout ffts_rope_pool writes and an HF cache stores), once per KV head for
// all G q-heads of its group: HBM-bound at 2 * B * Hkv * Lk * D * 2 bytes.
//
// decode_split_kernel: CTA = (b, kv head, split of the keys); 128 threads.  The
// split's keys are walked in chunks of 128:
//   scores   thread = key; 16-byte loads of the key's row; q of the G heads in
//            shared memory (broadcast reads); fp32 dot products, in log2 units;
//   softmax  warp w handles heads w, w + 4, ...: chunk max, running max m and
//            sum l, the chunk's exponentials in place;
//   P V      thread = output dimension; V rows read coalesced; G accumulators,
//            rescaled when the running max moves.
// An optional additive bias per (sequence, key) -- the caller's attention mask,
// added to the scaled scores before the softmax as at pred.py:311-313 -- is
// read once per key with the key's scores.  Fully masked chunks contribute
// nothing (their maxima stay -inf and their exponentials are 0).
// The split's (o[D], m, l) per head go to a workspace.
// decode_merge_kernel: CTA = (b, q head): o = sum_s 2^(m_s - M) o_s /
// sum_s 2^(m_s - M) l_s, rounded to bf16.
// No waits; every __syncthreads is reached by the whole CTA; every index is
// bounded by Lk, G <= 16 and D = 128.

#include "ffts_common.cuh"

namespace ffts {
namespace decode {

constexpr int kD = 128;
constexpr int kThreads = 128;
constexpr int kChunk = 128;  // one key per thread in the score phase
constexpr int kMaxG = 16;

struct Params {
  const __nv_bfloat16 *q;  // [B, H, D] with strides qs_b, qs_h (unit over D)
  const __nv_bfloat16 *k, *v;
  int64_t qs_b, qs_h;
  int64_t ks_b, ks_h, ks_l;  // cache strides (elements)
  int64_t vs_b, vs_h, vs_l;
  int B, H, Hkv, Lk, splits, per_split;
  float scale_log2;
  float *ws;  // [B * Hkv, splits, G, D + 2]: o, m, l
  const void *bias;    // additive mask [B, Lk] (row stride bias_sb), fp32 or bf16; nullptr = none
  int bias_bf16;
  int64_t bias_sb;
};

__device__ __forceinline__ float bias_log2(const Params &p, int b, int key) {
  if (p.bias == nullptr) return 0.0f;
  const int64_t i = int64_t(b) * p.bias_sb + key;
  const float x = p.bias_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(p.bias)[i])
                              : static_cast<const float *>(p.bias)[i];
  return x * 1.4426950408889634f;  // scores are kept in log2 units
}

__global__ void __launch_bounds__(kThreads) decode_split_kernel(const __grid_constant__ Params p) {
  __shared__ float q_s[kMaxG][kD];
  __shared__ float s_s[kMaxG][kChunk];
  __shared__ float m_s[kMaxG], l_s[kMaxG], a_s[kMaxG];
  const int G = p.H / p.Hkv;
  const int bh = blockIdx.x;  // b * Hkv + kv head
  const int b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int split = blockIdx.y;
  const int t = threadIdx.x;
  const int k0 = split * p.per_split;
  const int k1 = min(p.Lk, k0 + p.per_split);
  for (int i = t; i < G * kD; i += kThreads) {
    const int g = i / kD, d = i % kD;
    q_s[g][d] = __bfloat162float(p.q[int64_t(b) * p.qs_b + int64_t(kvh * G + g) * p.qs_h + d]);
  }
  if (t < G) {
    m_s[t] = -INFINITY;
    l_s[t] = 0.0f;
  }
  float acc[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) acc[g] = 0.0f;
  const __nv_bfloat16 *kb = p.k + int64_t(b) * p.ks_b + int64_t(kvh) * p.ks_h;
  const __nv_bfloat16 *vb = p.v + int64_t(b) * p.vs_b + int64_t(kvh) * p.vs_h;
  __syncthreads();
  for (int c0 = k0; c0 < k1; c0 += kChunk) {
    const int n = min(kChunk, k1 - c0);
    if (t < n) {
      const __nv_bfloat16 *row = kb + int64_t(c0 + t) * p.ks_l;
      float dot[kMaxG];
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) dot[g] = 0.0f;
#pragma unroll 4
      for (int d0 = 0; d0 < kD; d0 += 8) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(row + d0);
        const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < kMaxG; ++g) {
          if (g < G) {
#pragma unroll
            for (int e = 0; e < 8; ++e) dot[g] = fmaf(q_s[g][d0 + e], kf[e], dot[g]);
          }
        }
      }
      const float bl = bias_log2(p, b, c0 + t);
#pragma unroll
      for (int g = 0; g < kMaxG; ++g)
        if (g < G) s_s[g][t] = fmaf(dot[g], p.scale_log2, bl);
    }
    __syncthreads();
    const int warp = t >> 5, lane = t & 31;
    for (int g = warp; g < G; g += kThreads / 32) {
      float mx = -INFINITY;
      for (int i = lane; i < n; i += 32) mx = fmaxf(mx, s_s[g][i]);
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = m_s[g];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
      for (int i = lane; i < n; i += 32) {
        const float e = m_new == -INFINITY ? 0.0f : exp2f(s_s[g][i] - m_new);
        s_s[g][i] = e;
        sum += e;
      }
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.0f : exp2f(m_old - m_new);
        a_s[g] = alpha;
        l_s[g] = l_s[g] * alpha + sum;
        m_s[g] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kMaxG; ++g)
      if (g < G) acc[g] *= a_s[g];
    for (int i = 0; i < n; ++i) {
      const float vv = __bfloat162float(vb[int64_t(c0 + i) * p.vs_l + t]);
#pragma unroll
      for (int g = 0; g < kMaxG; ++g)
        if (g < G) acc[g] = fmaf(s_s[g][i], vv, acc[g]);
    }
    __syncthreads();
  }
  float *w = p.ws + (int64_t(bh) * p.splits + split) * G * (kD + 2);
#pragma unroll
  for (int g = 0; g < kMaxG; ++g)
    if (g < G) w[g * (kD + 2) + t] = acc[g];
  if (t < G) {
    w[t * (kD + 2) + kD] = m_s[t];
    w[t * (kD + 2) + kD + 1] = l_s[t];
  }
}

__global__ void __launch_bounds__(kThreads) decode_merge_kernel(const __grid_constant__ Params p,
                                                                __nv_bfloat16 *out, int64_t os_b, int64_t os_h) {
  const int G = p.H / p.Hkv;
  const int bhq = blockIdx.x;  // b * H + q head
  const int b = bhq / p.H, h = bhq % p.H;
  const int kvh = h / G, g = h % G;
  const int t = threadIdx.x;
  const float *w = p.ws + (int64_t(b) * p.Hkv + kvh) * p.splits * G * (kD + 2) + int64_t(g) * (kD + 2);
  const int64_t step = int64_t(G) * (kD + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, w[s * step + kD]);
  float num = 0.0f, den = 0.0f;
  for (int s = 0; s < p.splits; ++s) {
    const float ms = w[s * step + kD];
    if (ms == -INFINITY) continue;
    const float f = exp2f(ms - M);
    num = fmaf(f, w[s * step + t], num);
    den = fmaf(f, w[s * step + kD + 1], den);
  }
  out[int64_t(b) * os_b + int64_t(h) * os_h + t] = __float2bfloat16_rn(den > 0.0f ? num / den : 0.0f);
}

}  // namespace decode

int64_t decode_workspace_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t splits) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || splits <= 0) return 0;
  return B * Hkv * splits * (H / Hkv) * (decode::kD + 2) * 4;
}

int decode_attn(const void *q, int64_t qs_b, int64_t qs_h, const void *k, const int64_t *ks, const void *v,
                const int64_t *vs, int64_t B, int64_t H, int64_t Hkv, int64_t Lk, int64_t D, int64_t splits,
                void *ws, int64_t ws_bytes, void *out, int64_t os_b, int64_t os_h, const void *bias,
                int bias_dtype, int64_t bias_sb, cudaStream_t stream) {
  using namespace decode;
  FFTS_REQUIRE(q && k && v && ks && vs && ws && out, "decode: NULL argument");
  FFTS_REQUIRE(D == kD, "decode: head_dim must be 128 (got %lld)", (long long)D);
  FFTS_REQUIRE(B >= 1 && H >= 1 && Hkv >= 1 && H % Hkv == 0 && H / Hkv <= kMaxG && Lk >= 1 && splits >= 1,
               "decode: bad shape (B %lld, H %lld, Hkv %lld, Lk %lld, splits %lld; at most %d q-heads per KV head)",
               (long long)B, (long long)H, (long long)Hkv, (long long)Lk, (long long)splits, kMaxG);
  FFTS_REQUIRE(Lk < (int64_t(1) << 31) && B * Hkv <= 0x7fffffff && B * H <= 0x7fffffff, "decode: shape too large");
  FFTS_REQUIRE(ks[2] % 8 == 0 && ks[2] >= D && vs[2] >= D,
               "decode: cache row strides must be at least D (the key cache's a multiple of 8 elements)");
  FFTS_REQUIRE((reinterpret_cast<uintptr_t>(k) & 15) == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0 &&
                   ks[0] % 8 == 0 && ks[1] % 8 == 0,
               "decode: the key cache must be 16-byte aligned");
  const int64_t per = ceil_div(Lk, splits);
  const int64_t nsplit = ceil_div(Lk, per);  // every split non-empty
  FFTS_REQUIRE(nsplit <= 65535, "decode: too many splits");
  FFTS_REQUIRE(ws_bytes >= decode_workspace_bytes(B, H, Hkv, nsplit), "decode: workspace too small");
  Params p{};
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.k = static_cast<const __nv_bfloat16 *>(k);
  p.v = static_cast<const __nv_bfloat16 *>(v);
  p.qs_b = qs_b;
  p.qs_h = qs_h;
  p.ks_b = ks[0];
  p.ks_h = ks[1];
  p.ks_l = ks[2];
  p.vs_b = vs[0];
  p.vs_h = vs[1];
  p.vs_l = vs[2];
  p.B = int(B);
  p.H = int(H);
  p.Hkv = int(Hkv);
  p.Lk = int(Lk);
  p.per_split = int(per);
  p.splits = int(nsplit);
  p.scale_log2 = float(1.4426950408889634 / sqrt(double(D)));
  p.ws = static_cast<float *>(ws);
  FFTS_REQUIRE(bias == nullptr || bias_dtype == FFTS_DTYPE_F32 || bias_dtype == FFTS_DTYPE_BF16,
               "decode: the additive mask must be fp32 or bf16");
  FFTS_REQUIRE(bias == nullptr || B == 1 || bias_sb >= Lk, "decode: mask row stride %lld shorter than Lk %lld",
               (long long)bias_sb, (long long)Lk);
  p.bias = bias;
  p.bias_bf16 = bias_dtype == FFTS_DTYPE_BF16 ? 1 : 0;
  p.bias_sb = bias_sb;
  decode_split_kernel<<<dim3(unsigned(B * Hkv), unsigned(nsplit)), kThreads, 0, stream>>>(p);
  FFTS_CUDA(cudaGetLastError());
  decode_merge_kernel<<<unsigned(B * H), kThreads, 0, stream>>>(p, static_cast<__nv_bfloat16 *>(out), os_b, os_h);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
