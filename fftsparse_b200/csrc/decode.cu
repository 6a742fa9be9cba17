// decode.cu -- single-token decode attention over a head-major KV cache.
//
// Replaces the caller's eager decode branch (eval/LongBench/pred.py:306-322:
// softmax(q k^T / sqrt(D)) v over the whole cache with repeat_kv-expanded k/v,
// fp32 softmax).  It reads the cache un-expanded, [B, Hkv, Lk, D] bf16 (the
// layout ffts_rope_pool writes and an HF cache stores), once per KV head for
// all G q-heads of its group: HBM-bound at 2 * B * Hkv * Lk * D * 2 bytes.
//
// decode_split_kernel: CTA = (b, kv head, split of the keys, up to 8 q-heads
// of the group); 256 threads; two CTAs per SM with 3-stage rings when a CTA
// holds up to 4 heads, one with 4 stages for 8 heads (registers).  The split's
// keys are cut into chunks of 8 rows; warp w takes chunks w, w + 8, ... and
// streams their K and V rows through its own cp.async ring, so about 128 KB of
// cache per SM is in flight and no CTA-wide barrier interrupts the stream:
//   scores   a half-warp per key row (lane = 8 channels, 16 bytes), q of the
//            heads in registers; fp32 dot products reduced over the 16 lanes,
//            in log2 units;
//   softmax  per warp and head: running max m and sum l, updated per chunk;
//   P V      each lane accumulates its 8 channels for every head, rescaled when
//            the running max moves.
// An optional additive bias per (sequence, key) -- the caller's attention mask,
// added to the scaled scores before the softmax as at pred.py:311-313 -- is
// read once per key with the key's scores.  Fully masked keys contribute
// nothing (their exponentials are 0).  At the end of the split the warps'
// (o[D], m, l) are rescaled to their common maximum and summed into the
// workspace.
// decode_merge_kernel: CTA = (b, q head): o = sum_s 2^(m_s - M) o_s /
// sum_s 2^(m_s - M) l_s, rounded to bf16.
// No spin-waits (cp.async completion is a hardware wait on the warp's own
// copies); every __syncthreads is reached by the whole CTA; every index is
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
  const int64_t i = int64_t(b) * p.bias_sb + FFTS_INDEX(key, p.Lk);
  const float x = p.bias_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(p.bias)[i])
                              : static_cast<const float *>(p.bias)[i];
  return x * 1.4426950408889634f;  // scores are kept in log2 units
}

constexpr int kSplitThreads = 256;  // 8 warps, each walking its own chunks of keys
constexpr int kWarps = kSplitThreads / 32;
constexpr int kHeadsPerCta = 8;     // q-heads of one group per CTA (groups of up to 16 take two CTAs)

__device__ __forceinline__ void widen8(const uint4 &raw, float *f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// 16-byte global -> shared copy; src_bytes 0 writes zeros without reading
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Dynamic shared memory of decode_split_kernel<GM, ITS, NS, MINB>: every warp's
// ring of NS chunks, K rows then V rows of 2 * ITS keys (256 bytes each).
template <int ITS, int NS>
constexpr int split_smem_bytes() {
  return kWarps * NS * 2 * (2 * ITS) * kD * 2;
}

// CTA = (b, kv head, split of the keys, block of up to 8 q-heads of the group);
// 256 threads.  The split's keys are cut into chunks of R = 2 * ITS rows, and
// warp w takes chunks w, w + 8, ...: each warp keeps its own online softmax
// (running max m and sum l per head, in log2 units) and P V accumulators, so
// warps never wait for one another until the end of the split.  A warp's K and
// V rows stream through its own kStages-deep cp.async ring: a half-warp copies
// one 256-byte row (lane = 16 bytes, 8 channels) and later reads back exactly
// the bytes it copied, so no cross-lane barrier is needed.  Per chunk: the GM
// dot products of a row are reduced over the half-warp's 16 lanes together
// (log2 GM halving exchanges leave each lane one head's score, 5 shuffles for
// 4 heads where one reduction per head would take 16); that lane runs the head's
// online softmax; each lane then accumulates P V for its 8 channels and every
// head, with the heads' p and rescale factors taken from their lanes, in paired
// fp32 FMAs.  At the end the halves, then the warps (rescaled to the
// CTA's maximum) are summed into the split's (o, m, l) per head.
template <int GM, int ITS, int kStages, int MINB>
__global__ void __launch_bounds__(kSplitThreads, MINB) decode_split_kernel(const __grid_constant__ Params p) {
  constexpr int R = 2 * ITS;
  constexpr int kRowBytes = kD * 2;
  constexpr int kSlot = 2 * R * kRowBytes;  // K rows, then V rows
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ float wm[kWarps][GM], wl[kWarps][GM];
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
  // q of this CTA's heads for the lane's 8 channels (as 4 pairs), pre-multiplied by scale * log2(e)
  float2 q2[GM][4];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    float f[8];
    if (g < ng) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(p.q + int64_t(b) * p.qs_b +
                                                         int64_t(kvh * G + g0 + g) * p.qs_h + seg * 8);
      widen8(raw, f);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) q2[g][j] = make_float2(f[2 * j] * p.scale_log2, f[2 * j + 1] * p.scale_log2);
  }
  // After the reduction below, lane seg of each half holds the score of head hl
  // (the sums of the GM heads are split over the 16 lanes, LG = log2(GM) bits of
  // seg); that lane keeps the running max m and sum l of head hl, the same in
  // every lane of the head and in both halves.
  constexpr int LG = GM == 1 ? 0 : (GM == 2 ? 1 : (GM == 4 ? 2 : 3));
  const int hl = LG ? (seg >> (4 - LG)) : 0;
  const bool head_ok = hl < ng;
  float m = -INFINITY, l = 0.0f;
  float2 acc[GM][4];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[g][j] = make_float2(0.0f, 0.0f);
  const __nv_bfloat16 *kb = p.k + int64_t(b) * p.ks_b + int64_t(kvh) * p.ks_h + seg * 8;
  const __nv_bfloat16 *vb = p.v + int64_t(b) * p.vs_b + int64_t(kvh) * p.vs_h + seg * 8;
  const uint32_t ring = static_cast<uint32_t>(__cvta_generic_to_shared(dsm)) + uint32_t(warp * kStages * kSlot);
  const uint8_t *ring_p = dsm + warp * kStages * kSlot;
  // the lane's 16 bytes of row 2 * it + half inside a slot's K (V: + R rows)
  const uint32_t lane_off = uint32_t(half * kRowBytes + seg * 16);
  const int nchunks = (k1 - k0 + R - 1) / R;
  const int mine = nchunks > warp ? (nchunks - warp + kWarps - 1) / kWarps : 0;  // chunks of this warp

  auto issue = [&](int j) {  // this warp's chunk j into slot j % kStages
    const int base = k0 + (warp + kWarps * j) * R;
    const uint32_t slot = ring + uint32_t((j % kStages) * kSlot) + lane_off;
#pragma unroll
    for (int it = 0; it < ITS; ++it) {
      const int row = base + 2 * it + half;
      const bool ok = row < k1;
      const int64_t r = ok ? FFTS_INDEX(row, p.Lk) : k0;  // a valid address; nothing is read when !ok
      cp_async16(slot + uint32_t(2 * it * kRowBytes), kb + r * p.ks_l, ok ? 16 : 0);
      cp_async16(slot + uint32_t((R + 2 * it) * kRowBytes), vb + r * p.vs_l, ok ? 16 : 0);
    }
  };
#pragma unroll
  for (int j = 0; j < kStages - 1; ++j) {
    if (j < mine) issue(j);
    cp_async_commit();  // empty groups keep the count uniform
  }
  for (int j = 0; j < mine; ++j) {
    if (j + kStages - 1 < mine) issue(j + kStages - 1);
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // chunk j has landed (this lane's own bytes)
    const uint8_t *slot = ring_p + (j % kStages) * kSlot + lane_off;
    const int base = k0 + (warp + kWarps * j) * R;
    // ---- scores of the chunk's rows (this half's rows: 2 * it + half)
    float sc[ITS];
#pragma unroll
    for (int it = 0; it < ITS; ++it) {
      const int row = base + 2 * it + half;
      float kf[8];
      widen8(*reinterpret_cast<const uint4 *>(slot + 2 * it * kRowBytes), kf);
      float part[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < 4; ++j) a = __ffma2_rn(q2[g][j], make_float2(kf[2 * j], kf[2 * j + 1]), a);
        part[g] = a.x + a.y;
      }
      // reduce the GM partial sums over the 16 lanes together: while more than one
      // value is held, each exchange step keeps the lower or upper half of the heads
      // (by the lane's bit) and adds the partner's share of them
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        const int mask = 8 >> st;
        const int n = GM >> st;
        if (n >= 2) {
          const bool up = (seg & mask) != 0;
#pragma unroll
          for (int jj = 0; jj < GM / 2; ++jj) {
            if (jj < n / 2) {
              const float send = up ? part[jj] : part[jj + n / 2];
              const float keep = up ? part[jj + n / 2] : part[jj];
              part[jj] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
            }
          }
        } else {
          part[0] += __shfl_xor_sync(0xffffffffu, part[0], mask);
        }
      }
      const float bl = row < k1 ? bias_log2(p, b, row) : 0.0f;
      sc[it] = (row < k1 && head_ok) ? part[0] + bl : -INFINITY;
    }
    // ---- online softmax of head hl over the chunk (the halves combine)
    float mx = sc[0];
#pragma unroll
    for (int it = 1; it < ITS; ++it) mx = fmaxf(mx, sc[it]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float m_new = fmaxf(m, mx);
    const float alpha = m_new == -INFINITY ? 1.0f : exp2f(m - m_new);
    float pr[ITS];
    float sum = 0.0f;
#pragma unroll
    for (int it = 0; it < ITS; ++it) {
      pr[it] = m_new == -INFINITY ? 0.0f : exp2f(sc[it] - m_new);
      sum += pr[it];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 16);
    l = l * alpha + sum;
    m = m_new;
    // ---- P V for the lane's 8 channels, every head: alpha and p from the head's lanes
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      const float ag = __shfl_sync(0xffffffffu, alpha, g << (4 - LG));
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] = __fmul2_rn(acc[g][j], make_float2(ag, ag));
    }
#pragma unroll
    for (int it = 0; it < ITS; ++it) {
      float vf[8];
      widen8(*reinterpret_cast<const uint4 *>(slot + (R + 2 * it) * kRowBytes), vf);
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const float pg = __shfl_sync(0xffffffffu, pr[it], (half << 4) | (g << (4 - LG)));
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[g][j] = __ffma2_rn(make_float2(pg, pg), make_float2(vf[2 * j], vf[2 * j + 1]), acc[g][j]);
      }
    }
  }
  cp_async_wait<0>();
  // ---- the two halves of the warp hold the same channels of different rows
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[g][j].x += __shfl_xor_sync(0xffffffffu, acc[g][j].x, 16);
      acc[g][j].y += __shfl_xor_sync(0xffffffffu, acc[g][j].y, 16);
    }
  __syncthreads();  // every warp is done with its ring: reuse it for the cross-warp sum
  float *red = reinterpret_cast<float *>(dsm);  // [kWarps][GM][kD]
  if (half == 0) {
#pragma unroll
    for (int g = 0; g < GM; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float2 *>(red + (warp * GM + g) * kD + seg * 8 + 2 * j) = acc[g][j];
  }
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    const float mg = __shfl_sync(0xffffffffu, m, g << (4 - LG));
    const float lgs = __shfl_sync(0xffffffffu, l, g << (4 - LG));
    if (lane == 0) {
      wm[warp][g] = mg;
      wl[warp][g] = lgs;
    }
  }
  __syncthreads();
  float *w = p.ws + (int64_t(bh) * p.splits + split) * G * (kD + 2);
  for (int idx = tid; idx < ng * kD; idx += kSplitThreads) {
    const int g = idx / kD, d = idx % kD;
    float M = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < kWarps; ++ww) M = fmaxf(M, wm[ww][g]);
    float o = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kWarps; ++ww)
      if (wm[ww][g] != -INFINITY) o = fmaf(exp2f(wm[ww][g] - M), red[(ww * GM + g) * kD + d], o);
    if (FFTS_IN_RANGE(g0 + g, G)) w[(g0 + g) * (kD + 2) + d] = o;
  }
  if (tid < ng && FFTS_IN_RANGE(g0 + tid, G)) {
    float M = -INFINITY, L = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kWarps; ++ww) M = fmaxf(M, wm[ww][tid]);
#pragma unroll
    for (int ww = 0; ww < kWarps; ++ww)
      if (wm[ww][tid] != -INFINITY) L = fmaf(exp2f(wm[ww][tid] - M), wl[ww][tid], L);
    w[(g0 + tid) * (kD + 2) + kD] = M;
    w[(g0 + tid) * (kD + 2) + kD + 1] = L;
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

template <int GM, int ITS, int NS, int MINB>
static int launch_split(dim3 grid, const Params &p, cudaStream_t stream) {
  constexpr int smem = split_smem_bytes<ITS, NS>();
  static_assert(smem >= kWarps * GM * kD * 4, "the ring must hold the cross-warp sum");
  static_assert(MINB * (smem + 2048) <= 228 * 1024, "the CTAs of an SM must fit its shared memory");
  int rc = ensure_func_smem(reinterpret_cast<const void *>(&decode_split_kernel<GM, ITS, NS, MINB>), smem,
                           int(cudaSharedmemCarveoutMaxShared));
  if (rc) return rc;
  decode_split_kernel<GM, ITS, NS, MINB><<<grid, kSplitThreads, smem, stream>>>(p);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
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
  // chunks of 8 keys per warp
  int rc = FFTS_OK;
  // up to 4 heads per CTA: two CTAs per SM with 3-stage rings; 8 heads: one, 4 stages
  if (gm <= 1)
    rc = launch_split<1, 4, 3, 2>(grid, p, stream);
  else if (gm <= 2)
    rc = launch_split<2, 4, 3, 2>(grid, p, stream);
  else if (gm <= 4)
    rc = launch_split<4, 4, 3, 2>(grid, p, stream);
  else
    rc = launch_split<8, 4, 4, 1>(grid, p, stream);
  if (rc) return rc;
  decode_merge_kernel<<<unsigned(B * H), kThreads, 0, stream>>>(p, static_cast<__nv_bfloat16 *>(out), os_b, os_h);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
