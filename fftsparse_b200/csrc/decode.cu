// decode.cu -- single-token decode attention over a head-major KV cache.
//
// Replaces the caller's eager decode branch (eval/LongBench/pred.py:306-322:
// softmax(q k^T / sqrt(D)) v over the whole cache with repeat_kv-expanded k/v,
// fp32 softmax).  It reads the cache un-expanded, [B, Hkv, Lk, D] bf16 (the
// layout ffts_rope_pool writes and an HF cache stores), once per KV head for
// all G q-heads of its group: HBM-bound at 2 * B * Hkv * Lk * D * 2 bytes.
//
// decode_split_kernel: CTA = (b, kv head, split of the keys, up to 8 q-heads
// of the group); 256 threads.  The split's keys are walked in chunks of 64:
//   scores   a half-warp per key row, 16-byte loads (lane = 8 channels), so each
//            warp instruction reads two whole rows; q of the heads in
//            registers; fp32 dot products reduced over the 16 lanes, in log2
//            units;
//   softmax  warp w handles head w: chunk max, running max m and sum l, the
//            chunk's exponentials in place;
//   P V      the same row split over V; each lane accumulates its 8 channels for
//            every head, rescaled when the running max moves; the row slots
//            are summed once at the end of the split.
// An optional additive bias per (sequence, key) -- the caller's attention mask,
// added to the scaled scores before the softmax as at pred.py:311-313 -- is
// read once per key with the key's scores.  Fully masked chunks contribute
// nothing (their maxima stay -inf and their exponentials are 0).
// The split's (o[D], m, l) per head go to a workspace.
// decode_merge_kernel: CTA = (b, q head): o = sum_s 2^(m_s - M) o_s /
// sum_s 2^(m_s - M) l_s, rounded to bf16.
// No waits; every __syncthreads is reached by the whole CTA; every index is
// bounded by Lk, G <= 16 (in blocks of 8 heads per CTA) and D = 128.

#include <algorithm>

#include "ffts_common.cuh"

namespace ffts {
namespace decode {

constexpr int kD = 128;
constexpr int kThreads = 128;
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

constexpr int kSplitThreads = 256;  // 8 warps
constexpr int kRows = 64;           // keys per chunk: 8 per warp, two per warp instruction
constexpr int kHeadsPerCta = 8;     // q-heads of one group per CTA (groups of up to 16 take two CTAs)

__device__ __forceinline__ void widen8(const uint4 &raw, float *f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// CTA = (b, kv head, split of the keys, block of up to 8 q-heads of the group);
// 256 threads.  Each half-warp reads one key row with 16-byte loads (lane =
// 8-channel segment), so a warp instruction moves two whole 256-byte rows and a
// chunk of 64 rows is in flight per CTA; the G dot products of a row are
// reduced over the 16 lanes by shuffles.  Softmax per chunk as before (warp w
// handles head w); P V: each lane accumulates its 8 channels over its rows for
// every head, and the 16 row slots are summed once at the end of the split.
template <int GM>
__global__ void __launch_bounds__(kSplitThreads) decode_split_kernel(const __grid_constant__ Params p) {
  __shared__ float s_s[GM][kRows];
  __shared__ float m_s[GM], l_s[GM], a_s[GM];
  __shared__ float red[kSplitThreads / 32][GM][kD];
  const int G = p.H / p.Hkv;
  const int bh = blockIdx.x;  // b * Hkv + kv head
  const int b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int split = blockIdx.y;
  const int g0 = blockIdx.z * kHeadsPerCta;
  const int ng = min(GM, G - g0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = lane >> 4, seg = lane & 15;
  const int k0 = split * p.per_split;
  const int k1 = min(p.Lk, k0 + p.per_split);
  // q of this CTA's heads for the lane's 8 channels, pre-multiplied by scale * log2(e)
  float qr[GM][8];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < ng) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(p.q + int64_t(b) * p.qs_b +
                                                         int64_t(kvh * G + g0 + g) * p.qs_h + seg * 8);
      widen8(raw, qr[g]);
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[g][e] *= p.scale_log2;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[g][e] = 0.0f;
    }
  }
  if (tid < GM) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.0f;
  }
  float acc[GM][8];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.0f;
  const __nv_bfloat16 *kb = p.k + int64_t(b) * p.ks_b + int64_t(kvh) * p.ks_h + seg * 8;
  const __nv_bfloat16 *vb = p.v + int64_t(b) * p.vs_b + int64_t(kvh) * p.vs_h + seg * 8;
  __syncthreads();
  for (int c0 = k0; c0 < k1; c0 += kRows) {
    const int n = min(kRows, k1 - c0);
    // rows warp * 8 + 2 * it + half of the chunk: K and V loads issued together
    uint4 kv[4], vv[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int row = warp * 8 + 2 * it + half;
      kv[it] = row < n ? *reinterpret_cast<const uint4 *>(kb + int64_t(c0 + row) * p.ks_l) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int row = warp * 8 + 2 * it + half;
      vv[it] = row < n ? *reinterpret_cast<const uint4 *>(vb + int64_t(c0 + row) * p.vs_l) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int row = warp * 8 + 2 * it + half;
      float kf[8];
      widen8(kv[it], kf);
      const float bl = (seg == 0 && row < n) ? bias_log2(p, b, c0 + row) : 0.0f;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        float part = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) part = fmaf(qr[g][e], kf[e], part);
#pragma unroll
        for (int o = 8; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (seg == 0 && row < n) s_s[g][row] = part + bl;
      }
    }
    __syncthreads();
    // softmax of the chunk: warp w handles head w
    if (warp < ng) {
      const int g = warp;
      const float x = lane < n ? s_s[g][lane] : -INFINITY;
      const float y = lane + 32 < n ? s_s[g][lane + 32] : -INFINITY;
      float mx = fmaxf(x, y);
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = m_s[g];
      const float m_new = fmaxf(m_old, mx);
      const float ex = m_new == -INFINITY ? 0.0f : exp2f(x - m_new);
      const float ey = m_new == -INFINITY ? 0.0f : exp2f(y - m_new);
      s_s[g][lane] = ex;
      s_s[g][lane + 32] = ey;
      float sum = ex + ey;
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.0f : exp2f(m_old - m_new);
        a_s[g] = alpha;
        l_s[g] = l_s[g] * alpha + sum;
        m_s[g] = m_new;
      }
    }
    __syncthreads();
    // P V over the same rows
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      const float alpha = g < ng ? a_s[g] : 1.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
    }
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int row = warp * 8 + 2 * it + half;
      float vf[8];
      widen8(vv[it], vf);
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const float pr = (g < ng && row < n) ? s_s[g][row] : 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(pr, vf[e], acc[g][e]);
      }
    }
    __syncthreads();  // s_s is rewritten by the next chunk
  }
  // sum the 16 row slots: the two halves of each warp, then the 8 warps
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], 16);
  if (half == 0) {
#pragma unroll
    for (int g = 0; g < GM; ++g)
#pragma unroll
      for (int e = 0; e < 8; ++e) red[warp][g][seg * 8 + e] = acc[g][e];
  }
  __syncthreads();
  float *w = p.ws + (int64_t(bh) * p.splits + split) * G * (kD + 2);
  for (int idx = tid; idx < ng * kD; idx += kSplitThreads) {
    const int g = idx / kD, d = idx % kD;
    float o = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kSplitThreads / 32; ++ww) o += red[ww][g][d];
    w[(g0 + g) * (kD + 2) + d] = o;
  }
  if (tid < ng) {
    w[(g0 + tid) * (kD + 2) + kD] = m_s[tid];
    w[(g0 + tid) * (kD + 2) + kD + 1] = l_s[tid];
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
  FFTS_REQUIRE(ks[2] >= D && vs[2] >= D && ks[0] % 8 == 0 && ks[1] % 8 == 0 && ks[2] % 8 == 0 &&
                   vs[0] % 8 == 0 && vs[1] % 8 == 0 && vs[2] % 8 == 0 && qs_b % 8 == 0 && qs_h % 8 == 0,
               "decode: q and cache strides must be multiples of 8 elements (16 bytes), cache rows at least D");
  FFTS_REQUIRE((reinterpret_cast<uintptr_t>(k) & 15) == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(q) & 15) == 0,
               "decode: q and the caches must be 16-byte aligned");
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
  const int G = int(H / Hkv);
  const dim3 grid(unsigned(B * Hkv), unsigned(nsplit), unsigned(ceil_div(int64_t(G), int64_t(kHeadsPerCta))));
  const int gm = std::min(G, kHeadsPerCta);
  if (gm <= 1)
    decode_split_kernel<1><<<grid, kSplitThreads, 0, stream>>>(p);
  else if (gm <= 2)
    decode_split_kernel<2><<<grid, kSplitThreads, 0, stream>>>(p);
  else if (gm <= 4)
    decode_split_kernel<4><<<grid, kSplitThreads, 0, stream>>>(p);
  else
    decode_split_kernel<8><<<grid, kSplitThreads, 0, stream>>>(p);
  FFTS_CUDA(cudaGetLastError());
  decode_merge_kernel<<<unsigned(B * H), kThreads, 0, stream>>>(p, static_cast<__nv_bfloat16 *>(out), os_b, os_h);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
