// mask.cu -- FFTSparse block-mask selection on sm_100a.
//
// Replaces the selection half of myattn_prefill (attn_src/fft_attn/my_attn_v7.py
// :532-641) with three launches that keep every decision on the device (the
// reference syncs the host at :273 and :597 and loops over sampled diagonals on
// the host at :342-357):
//
//   select_stage1_kernel  one launch for all independent per-head jobs:
//      fft_warp_body /    per (b, h, 8-channel chunk): zero-padded FFT of
//      fft_partial_body   z = q + i k per channel, cross spectrum Q conj(K)
//                         summed over the chunk's channels
//                         (batch_fft_cross_correlation, :117-131); a
//                         register-resident FFT, one warp per channel, for
//                         lengths up to 2048, else shared-memory butterflies;
//                         both compute the same butterflies;
//      diag_group_body    per (b, h, group of up to 8 sampled lags): the
//                         normalised variance of each lag's block-score
//                         diagonal (compute_stripe_variance, :301-383), with the
//                         q and k rows the group needs staged once;
//      colrow_body        per (b, h): hot key columns (create_column_block_mask,
//                         :390-447) and the last query row's top-k
//                         (create_last_block_query_mask, :54-72).
//   corr_select_kernel    per (b, h): the stripe decision, one inverse FFT of the
//                         summed spectrum, the post-processing (:132-155) and the
//                         lag selection (create_correlation_block_mask, :195-208).
//   mask_build_kernel     per (b, h, row tile): per-row QK top-k for diffuse
//                         heads (create_qk_topk_block_mask, :256-294) and the
//                         union with the prior, Toeplitz lag, column and last-row
//                         masks (:74-98, :212-225, :606-641) into packed bits.
//
// Arithmetic is the canonical one restated by oracle/ffts_oracle.c: fp32 FFT
// butterflies with no contraction (__fmul_rn/__fadd_rn), exact-product fp64
// dot products for block scores, fp64 reductions in a fixed 256-lane order, and
// top-k ties broken by lowest block index.

#include <math.h>
#include <stdarg.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "ffts_common.cuh"

namespace ffts {

// ---------------------------------------------------------------- tables
// Forward twiddles of the largest FFT: g_twiddle[j] = (cos a, -sin a) with
// a = 2*pi*j / kMaxFFT; an FFT of length M uses entry j * (kMaxFFT / M), which is
// bit-identical to evaluating a = 2*pi*j / M directly (power-of-two scaling).
__device__ float2 g_twiddle[kMaxFFT / 2];
// g_log10[n] = (float)log10(n), n <= kMaxBlocks
__device__ float g_log10[kMaxBlocks + 1];

static std::mutex g_table_mutex;
static std::vector<int> g_table_ready;

int ensure_tables() {
  int dev = 0;
  FFTS_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_table_mutex);
  if (dev < int(g_table_ready.size()) && g_table_ready[dev]) return FFTS_OK;
  std::vector<float2> tw(kMaxFFT / 2);
  for (int j = 0; j < kMaxFFT / 2; ++j) {
    const double a = (2.0 * M_PI * (double)j) / (double)kMaxFFT;
    tw[j] = make_float2((float)cos(a), (float)(-sin(a)));
  }
  std::vector<float> lg(kMaxBlocks + 1);
  lg[0] = -INFINITY;
  for (int n = 1; n <= kMaxBlocks; ++n) lg[n] = (float)log10((double)n);
  FFTS_CUDA(cudaMemcpyToSymbol(g_twiddle, tw.data(), tw.size() * sizeof(float2)));
  FFTS_CUDA(cudaMemcpyToSymbol(g_log10, lg.data(), lg.size() * sizeof(float)));
  if (dev >= int(g_table_ready.size())) g_table_ready.resize(dev + 1, 0);
  g_table_ready[dev] = 1;
  return FFTS_OK;
}

// ------------------------------------------------------------------- FFT
__device__ __forceinline__ uint32_t bitrev(uint32_t x, int bits) { return __brev(x) >> (32 - bits); }

// Spans h = 1..16 of a radix-2 DIT on a warp-held 32-element segment
// (lane = index bits 0..4).  The upper element of each pair forms t = w*b and
// sends it; the lower sends a; the lower keeps a + t, the upper a - t.
__device__ __forceinline__ void fft_warp_stages(float &re, float &im, int lane, int M,
                                                const float2 *tw, bool inverse) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
    const bool upper = lane & h;
    float sr = re, si = im;
    if (upper) {
      float2 w = tw[(lane & (h - 1)) * (M / (2 * h))];
      if (inverse) w.y = -w.y;
      const float p1 = __fmul_rn(w.x, re), p2 = __fmul_rn(w.y, im);
      const float p3 = __fmul_rn(w.x, im), p4 = __fmul_rn(w.y, re);
      sr = __fsub_rn(p1, p2);
      si = __fadd_rn(p3, p4);
    }
    const float rr = __shfl_xor_sync(0xffffffffu, sr, h);
    const float ri = __shfl_xor_sync(0xffffffffu, si, h);
    if (upper) {
      re = __fsub_rn(rr, sr);
      im = __fsub_rn(ri, si);
    } else {
      re = __fadd_rn(sr, rr);
      im = __fadd_rn(si, ri);
    }
  }
}

// nfft independent length-M transforms stored back to back in x (input in
// bit-reversed order, output in natural order).  All threads of the CTA call.
__device__ void fft_block(float2 *x, int M, int nfft, const float2 *tw, bool inverse) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int nseg = nfft * (M >> 5);
  for (int seg = warp; seg < nseg; seg += nwarps) {
    float2 v = x[seg * 32 + lane];
    fft_warp_stages(v.x, v.y, lane, M, tw, inverse);
    x[seg * 32 + lane] = v;
  }
  __syncthreads();
  const int half = M >> 1;
  const int lh = ilog2_ceil(half);
  for (int h = 32; h < M; h <<= 1) {
    const int lgh = ilog2_ceil(h);
    const int step = M / (2 * h);
    for (int b = threadIdx.x; b < nfft * half; b += blockDim.x) {
      const int f = b >> lh, bb = b & (half - 1);
      const int g = bb >> lgh, k = bb & (h - 1);
      float2 *X = x + f * M;
      const int ia = g * 2 * h + k, ib = ia + h;
      float2 w = tw[k * step];
      if (inverse) w.y = -w.y;
      const float2 bv = X[ib], av = X[ia];
      const float p1 = __fmul_rn(w.x, bv.x), p2 = __fmul_rn(w.y, bv.y);
      const float p3 = __fmul_rn(w.x, bv.y), p4 = __fmul_rn(w.y, bv.x);
      const float tr = __fsub_rn(p1, p2), ti = __fadd_rn(p3, p4);
      X[ia] = make_float2(__fadd_rn(av.x, tr), __fadd_rn(av.y, ti));
      X[ib] = make_float2(__fsub_rn(av.x, tr), __fsub_rn(av.y, ti));
    }
    __syncthreads();
  }
}

template <typename T>
__device__ void fft_partial_body(const T *__restrict__ qb, const T *__restrict__ kb, int H, int Hkv, int N,
                                 int D, int M, int nf, float2 *__restrict__ partial, int chunk, int nchunk,
                                 int bh, unsigned char *smem_raw) {
  float2 *tw = reinterpret_cast<float2 *>(smem_raw);  // [M/2]
  float2 *acc = tw + M / 2;                            // [M/2 + 1]
  float2 *buf = acc + (M / 2 + 1) + 1;                 // [nf][M] (16-byte aligned)
  const int F = M / 2 + 1;
  const int bits = ilog2_ceil(M);
  const int b = bh / H, h = bh % H;
  const T *q = qb + int64_t(bh) * N * D;
  const T *k = kb + (int64_t(b) * Hkv + h / (H / Hkv)) * N * D;
  const int stride = kMaxFFT / M;
  for (int j = threadIdx.x; j < M / 2; j += blockDim.x) tw[j] = g_twiddle[j * stride];
  for (int f = threadIdx.x; f < F; f += blockDim.x) acc[f] = make_float2(0.0f, 0.0f);
  const int d_lo = chunk * kDChunk, d_hi = min(D, d_lo + kDChunk);
  for (int d0 = d_lo; d0 < d_hi; d0 += nf) {
    const int nb = min(nf, d_hi - d0);
    __syncthreads();
    for (int e = threadIdx.x; e < nb * M; e += blockDim.x) {
      const int fi = e / M, t = e - fi * M;
      float2 z = make_float2(0.0f, 0.0f);
      if (t < N && FFTS_IN_RANGE(d0 + fi, D))
        z = make_float2(Elem<T>::to_f32(q[int64_t(t) * D + d0 + fi]), Elem<T>::to_f32(k[int64_t(t) * D + d0 + fi]));
      if (FFTS_IN_RANGE(fi * M + bitrev(t, bits), nf * M)) buf[fi * M + bitrev(t, bits)] = z;
    }
    __syncthreads();
    fft_block(buf, M, nb, tw, false);
    for (int f = threadIdx.x; f < F; f += blockDim.x) {
      float2 a2 = acc[f];
      const int g = (M - f) & (M - 1);
      for (int fi = 0; fi < nb; ++fi) {
        const float2 A = buf[fi * M + f], Bv = buf[fi * M + g];
        const float qr = __fmul_rn(0.5f, __fadd_rn(A.x, Bv.x));
        const float qi = __fmul_rn(0.5f, __fsub_rn(A.y, Bv.y));
        const float kr = __fmul_rn(0.5f, __fadd_rn(A.y, Bv.y));
        const float ki = __fmul_rn(0.5f, __fsub_rn(Bv.x, A.x));
        const float cr = __fadd_rn(__fmul_rn(qr, kr), __fmul_rn(qi, ki));
        const float ci = __fsub_rn(__fmul_rn(qi, kr), __fmul_rn(qr, ki));
        a2.x = __fadd_rn(a2.x, cr);
        a2.y = __fadd_rn(a2.y, ci);
      }
      acc[f] = a2;
    }
  }
  __syncthreads();
  float2 *out = partial + (int64_t(bh) * nchunk + chunk) * F;
  for (int f = threadIdx.x; f < F; f += blockDim.x) out[f] = acc[f];
}

static size_t fft_partial_smem(int M, int nf) { return size_t(M / 2 + M / 2 + 2 + size_t(nf) * M) * sizeof(float2); }

// ------------------------------------------------- register-resident FFT
// The same radix-2 decimation-in-time transforms and cross spectra as
// fft_partial_body (identical butterflies, twiddles and channel order, so the
// partial spectra are bit-identical), for M = 32 * R <= 2048 points held in
// registers: one warp per channel, element i of the bit-reversed sequence in
// lane i / R, register i % R.  Spans h < R pair registers of one lane; the five
// spans h >= R pair lanes (shuffles).  One CTA of 8 warps takes one (b, h,
// 8-channel chunk); the channels' cross spectra are summed in channel order
// through shared memory.  Twiddles are re-laid per span so that the lanes of a
// warp read them from consecutive shared-memory words.
__host__ __device__ constexpr int rev_bits(int x, int n) {
  int y = 0;
  for (int i = 0; i < n; ++i) y |= ((x >> i) & 1) << (n - 1 - i);
  return y;
}
__host__ __device__ constexpr int log2_exact(int x) { return x <= 1 ? 0 : 1 + log2_exact(x >> 1); }

__device__ __forceinline__ void butterfly(float &ar, float &ai, float &br, float &bi, float2 w) {
  const float p1 = __fmul_rn(w.x, br), p2 = __fmul_rn(w.y, bi);
  const float p3 = __fmul_rn(w.x, bi), p4 = __fmul_rn(w.y, br);
  const float tr = __fsub_rn(p1, p2), ti = __fadd_rn(p3, p4);
  br = __fsub_rn(ar, tr);
  bi = __fsub_rn(ai, ti);
  ar = __fadd_rn(ar, tr);
  ai = __fadd_rn(ai, ti);
}

static size_t fft_warp_smem_rt(int R, int N, size_t elem) {
  const size_t stage = size_t(2) * kDChunk * size_t(N) * elem;
  const size_t sums = size_t(kDChunk) * R * 17 * sizeof(float2);
  return size_t(32 * R) * sizeof(float2) + (stage > sums ? stage : sums);
}

template <typename T, int R>
__device__ void fft_warp_body(const T *__restrict__ qb, const T *__restrict__ kb, int H, int Hkv, int N, int D,
                              int nchunk, float2 *__restrict__ partial, int f, unsigned char *smem_raw) {
  constexpr int LR = log2_exact(R);
  constexpr int M = 32 * R;
  constexpr int F = M / 2 + 1;
  constexpr int PS = R * 17;  // padded per-channel stride of the cross-spectrum buffer
  float2 *tin = reinterpret_cast<float2 *>(smem_raw);  // [R]: span h < R, index h + k
  float2 *tx = tin + R;                                 // [31 R]: span R << j at R (2^j - 1), index r 2^j + m
  unsigned char *uni = reinterpret_cast<unsigned char *>(tx + 31 * R);
  T *qs = reinterpret_cast<T *>(uni);                   // [8][N] staged channels (then reused)
  T *ks = qs + kDChunk * N;
  float2 *cs = reinterpret_cast<float2 *>(uni);         // [8][R][17] cross spectra
  const int chunk = f % nchunk, bh = f / nchunk;
  const int b = bh / H, h = bh % H;
  const T *q = qb + int64_t(bh) * N * D + chunk * kDChunk;
  const T *k = kb + (int64_t(b) * Hkv + h / (H / Hkv)) * N * D + chunk * kDChunk;
  constexpr int stride = kMaxFFT / M;
  for (int e = threadIdx.x; e < R; e += blockDim.x) {
    if (e >= 1) {
      const int hh = 1 << (31 - __clz(e)), kk = e - hh;
      tin[e] = g_twiddle[kk * (M / (2 * hh)) * stride];
    }
  }
  for (int e = threadIdx.x; e < 31 * R; e += blockDim.x) {
    const int j = 31 - __clz(e / R + 1);
    const int loc = e - R * ((1 << j) - 1);
    const int r = loc >> j, m = loc & ((1 << j) - 1);
    tx[e] = g_twiddle[(r + R * m) * (M / (2 * (R << j))) * stride];
  }
  // stage the chunk's 8 channels of q and k, channel-major
  constexpr int V = Elem<T>::kVec;
  constexpr int NV = kDChunk / V;  // 16-byte vectors per row and tensor
  constexpr int U = 4;             // rows in flight per thread
  const int nstage = FFTS_IN_RANGE(chunk * kDChunk + kDChunk - 1, D) ? N : 0;  // the chunk's channels exist
  for (int base = threadIdx.x; base < nstage; base += U * blockDim.x) {
    uint4 qv[U][NV], kv[U][NV];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u * blockDim.x;
      if (t < N) {
#pragma unroll
        for (int c = 0; c < NV; ++c) {
          qv[u][c] = *reinterpret_cast<const uint4 *>(q + int64_t(t) * D + c * V);
          kv[u][c] = *reinterpret_cast<const uint4 *>(k + int64_t(t) * D + c * V);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u * blockDim.x;
      if (t < N) {
#pragma unroll
        for (int c0 = 0; c0 < NV; ++c0) {
          const T *qe = reinterpret_cast<const T *>(&qv[u][c0]);
          const T *ke = reinterpret_cast<const T *>(&kv[u][c0]);
#pragma unroll
          for (int c = 0; c < V; ++c) {
            qs[(c0 * V + c) * N + t] = qe[c];
            ks[(c0 * V + c) * N + t] = ke[c];
          }
        }
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lb = __brev(uint32_t(lane)) >> 27;
  float re[R], im[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int t = (rev_bits(r, LR) << 5) | lb;  // bit reversal of i = lane * R + r
    re[r] = t < N ? Elem<T>::to_f32(qs[warp * N + t]) : 0.0f;
    im[r] = t < N ? Elem<T>::to_f32(ks[warp * N + t]) : 0.0f;
  }
  __syncthreads();  // the staging buffer becomes the cross-spectrum buffer
#pragma unroll
  for (int sp = 0; sp < LR; ++sp) {
    const int hh = 1 << sp;
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (!(r & hh)) butterfly(re[r], im[r], re[r + hh], im[r + hh], tin[hh + (r & (hh - 1))]);
  }
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const int hl = 1 << j;
    const bool upper = lane & hl;
    const int m = lane & (hl - 1);
    const float2 *tw = tx + R * (hl - 1);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float sr = re[r], si = im[r];
      if (upper) {
        const float2 w = tw[r * hl + m];
        const float p1 = __fmul_rn(w.x, sr), p2 = __fmul_rn(w.y, si);
        const float p3 = __fmul_rn(w.x, si), p4 = __fmul_rn(w.y, sr);
        sr = __fsub_rn(p1, p2);
        si = __fadd_rn(p3, p4);
      }
      const float rr = __shfl_xor_sync(0xffffffffu, sr, hl);
      const float ri = __shfl_xor_sync(0xffffffffu, si, hl);
      if (upper) {
        re[r] = __fsub_rn(rr, sr);
        im[r] = __fsub_rn(ri, si);
      } else {
        re[r] = __fadd_rn(sr, rr);
        im[r] = __fadd_rn(si, ri);
      }
    }
  }
  // X[f] sits at f = lane * R + r; its mirror (M - f) mod M at lane 31 - lane,
  // register R - r (r > 0), or lane (32 - lane) mod 32, register 0 (r = 0)
  float2 *cw = cs + warp * PS;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int src = r == 0 ? ((32 - lane) & 31) : 31 - lane;
    const float br = __shfl_sync(0xffffffffu, re[r == 0 ? 0 : R - r], src);
    const float bi = __shfl_sync(0xffffffffu, im[r == 0 ? 0 : R - r], src);
    if (lane < 16 || (lane == 16 && r == 0)) {
      const float qr = __fmul_rn(0.5f, __fadd_rn(re[r], br));
      const float qi = __fmul_rn(0.5f, __fsub_rn(im[r], bi));
      const float kr = __fmul_rn(0.5f, __fadd_rn(im[r], bi));
      const float ki = __fmul_rn(0.5f, __fsub_rn(br, re[r]));
      const float cr = __fadd_rn(__fmul_rn(qr, kr), __fmul_rn(qi, ki));
      const float ci = __fsub_rn(__fmul_rn(qi, kr), __fmul_rn(qr, ki));
      cw[r * 17 + lane] = make_float2(cr, ci);
    }
  }
  __syncthreads();
  float2 *out = partial + (int64_t(bh) * nchunk + chunk) * F;
  for (int pos = threadIdx.x; pos < PS; pos += blockDim.x) {
    const int r = pos / 17, L = pos - r * 17;
    if (L == 16 && r != 0) continue;
    float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < kDChunk; ++w) {
      const float2 c = cs[w * PS + pos];
      a.x = __fadd_rn(a.x, c.x);
      a.y = __fadd_rn(a.y, c.y);
    }
    if (FFTS_IN_RANGE(L * R + r, F)) out[L * R + r] = a;
  }
}



// ------------------------------------------------------- block selection
// Ascending-rank selection of 32-bit keys (keys[0..n)) by 8-bit radix passes.
__device__ uint32_t block_select_rank(const uint32_t *keys, int n, int rank, int *hist, int *bc) {
  uint32_t prefix = 0, mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t kk = keys[i];
      if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 255], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // the first digit d whose running count passes `rank`, and the count below it
      // (the total when none does): lane l scans bins [8l, 8l + 8) after a warp
      // prefix sum of the lanes' totals
      const int lane = threadIdx.x;
      int c[8], tot = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = hist[lane * 8 + e];
        tot += c[e];
      }
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int excl = incl - tot;
      const unsigned ball = __ballot_sync(0xffffffffu, rank >= excl && rank < incl);
      const int src = ball ? __ffs(ball) - 1 : 31;
      if (lane == src) {
        int cc = excl, dsel = 255;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (cc + c[e] > rank) { dsel = lane * 8 + e; break; }
          cc += c[e];
        }
        bc[0] = dsel;
        bc[1] = cc;
      }
    }
    __syncthreads();
    rank -= bc[1];
    prefix |= uint32_t(bc[0]) << shift;
    mask |= 0xffu << shift;
    __syncthreads();
  }
  return prefix;
}

// Set in `words` (pre-zeroed, indexed by absolute position) the bits of the k
// largest keys among keys[lo..hi); ties are broken by lowest index.
__device__ void block_topk_bits(const uint32_t *keys, int lo, int hi, int k, uint32_t *words,
                                int *hist, int *bc) {
  const int n = hi - lo;
  if (n <= 0 || k <= 0) return;
  if (k >= n) {
    for (int j = lo + threadIdx.x; j < hi; j += blockDim.x) atomicOr(&words[j >> 5], 1u << (j & 31));
    __syncthreads();
    return;
  }
  const uint32_t T = block_select_rank(keys + lo, n, n - k, hist, bc);
  // number of keys strictly greater than T
  if (threadIdx.x == 0) bc[2] = 0;
  __syncthreads();
  int local = 0;
  for (int j = lo + threadIdx.x; j < hi; j += blockDim.x) local += keys[j] > T;
  for (int o = 16; o; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(&bc[2], local);
  __syncthreads();
  const int need = k - bc[2];
  // walk indices in order; equal keys take the first `need` slots
  int *wsum = hist;  // reuse: per-warp counts
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int base = 0;
  for (int c = lo; c < hi; c += blockDim.x) {
    const int j = c + threadIdx.x;
    const bool in = j < hi;
    const bool eq = in && keys[j] == T;
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    __syncthreads();
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    int before = base;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    before += __popc(bal & ((1u << lane) - 1));
    int tot = 0;
    for (int w = 0; w < nw; ++w) tot += wsum[w];
    if (in && (keys[j] > T || (eq && before < need))) atomicOr(&words[j >> 5], 1u << (j & 31));
    base += tot;
  }
  __syncthreads();
}

// -------------------------------------------------- correlation + lag select
// Stage 2, one CTA per (b, h): the stripe decision (average of the per-lag
// statistics in sample order, my_attn_v7.py:359-363), then the summed cross
// spectrum's inverse FFT, post-processing and lag selection.  With the lag mask
// off it writes is_stripe = 0 and zero lag scores / selections.
__global__ void __launch_bounds__(512) corr_select_kernel(const float2 *__restrict__ partial,
                                                          int nchunk, int N, int M,
                                                          ffts_mask_params p,
                                                          const double *__restrict__ nv,
                                                          int32_t *__restrict__ stripe_ws,
                                                          uint8_t *__restrict__ is_stripe_out,
                                                          float *__restrict__ stripe_var_out,
                                                          float *__restrict__ corr_out,
                                                          float *__restrict__ csum_out,
                                                          uint32_t *__restrict__ tausel) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float2 *tw = reinterpret_cast<float2 *>(smem_raw);  // [M/2]
  float2 *X = tw + M / 2;                             // [M]
  float *corr = reinterpret_cast<float *>(X + M);     // [N]
  uint32_t *keys = reinterpret_cast<uint32_t *>(corr + N);  // [N]
  __shared__ int hist[256];
  __shared__ int bc[4];
  __shared__ float red[32];
  __shared__ double nvs[FFTS_MAX_DIAG_SAMPLES];
  const int bh = blockIdx.x;
  const int F = M / 2 + 1;
  const int bits = ilog2_ceil(M);
  const int W = (N + 31) / 32;
  const int stride = kMaxFFT / M;
  // the per-lag statistics are loaded side by side, then summed in sample order by one thread
  const bool stripe_test = p.corr_on && !p.stripe_all_diffuse;
  if (stripe_test)
    for (int s = threadIdx.x; s < p.n_diag_samples; s += blockDim.x)
      nvs[FFTS_INDEX(s, FFTS_MAX_DIAG_SAMPLES)] = nv[int64_t(bh) * FFTS_MAX_DIAG_SAMPLES + s];
  __syncthreads();
  if (threadIdx.x == 0) {
    float svar = INFINITY;
    int stripe = 0;
    if (stripe_test) {
      double total = 0.0;
      for (int s = 0; s < p.n_diag_samples; ++s) total = __dadd_rn(total, nvs[FFTS_INDEX(s, FFTS_MAX_DIAG_SAMPLES)]);
      svar = __double2float_rn(__ddiv_rn(total, (double)p.n_diag_samples));
      stripe = svar <= p.stripe_threshold;
    }
    stripe_ws[bh] = stripe;
    if (is_stripe_out) is_stripe_out[bh] = (uint8_t)stripe;
    if (stripe_var_out) stripe_var_out[bh] = svar;
  }
  if (!p.corr_on) {
    for (int w = threadIdx.x; w < W; w += blockDim.x) tausel[int64_t(bh) * W + w] = 0u;
    for (int t = threadIdx.x; t < N; t += blockDim.x) {
      if (corr_out) corr_out[int64_t(bh) * N + t] = 0.0f;
      if (csum_out) csum_out[int64_t(bh) * N + t] = 0.0f;
    }
    return;
  }
  for (int j = threadIdx.x; j < M / 2; j += blockDim.x) tw[j] = g_twiddle[j * stride];
  const float2 *part = partial + int64_t(bh) * nchunk * F;
  for (int f = threadIdx.x; f < F; f += blockDim.x) {
    float2 s = make_float2(0.0f, 0.0f);
    for (int c0 = 0; c0 < nchunk; c0 += 8) {  // eight chunks' loads in flight, added in chunk order
      float2 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = c0 + u < nchunk ? part[int64_t(c0 + u) * F + f] : make_float2(0.0f, 0.0f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (c0 + u < nchunk) {
          s.x = __fadd_rn(s.x, v[u].x);
          s.y = __fadd_rn(s.y, v[u].y);
        }
      }
    }
    X[bitrev(f, bits)] = s;
    if (f > 0 && f < M / 2) X[bitrev(M - f, bits)] = make_float2(s.x, -s.y);
  }
  __syncthreads();
  fft_block(X, M, 1, tw, true);
  const float invM = 1.0f / (float)M;
  const int ex = p.exclude_tau, sraw = p.sink_tau_raw;
  const int s0 = sraw >= 0 ? sraw : max(0, N + sraw);
  for (int t = threadIdx.x; t < N; t += blockDim.x) {
    const float cs = __fmul_rn(X[t].x, invM);
    if (csum_out) csum_out[int64_t(bh) * N + t] = cs;
    float c = __fdiv_rn(cs, (float)(N - t));
    if (t < ex || t >= s0) c = 0.0f;
    corr[t] = c;
  }
  __syncthreads();
  if (ex < sraw) {
    float mn = INFINITY;
    for (int t = ex + threadIdx.x; t < sraw; t += blockDim.x) mn = fminf(mn, corr[FFTS_INDEX(t, N)]);
    for (int o = 16; o; o >>= 1) mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mn;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m2 = red[0];
      for (int w = 1; w < int(blockDim.x >> 5); ++w) m2 = fminf(m2, red[w]);
      red[0] = m2;
    }
    __syncthreads();
    mn = red[0];
    const float lden0 = g_log10[FFTS_INDEX(N - ex, kMaxBlocks + 1)];
    const float lden = lden0 > 1e-6f ? lden0 : 1e-6f;
    for (int t = ex + threadIdx.x; t < sraw; t += blockDim.x) {
      const float w = __fdiv_rn(g_log10[FFTS_INDEX(N - t, kMaxBlocks + 1)], lden);
      if (FFTS_IN_RANGE(t, N)) corr[t] = __fmul_rn(__fsub_rn(corr[t], mn), w);
    }
    __syncthreads();
  }
  if (corr_out)
    for (int t = threadIdx.x; t < N; t += blockDim.x) corr_out[int64_t(bh) * N + t] = corr[t];

  // lag selection over the remote range [rs, N)
  const int rs = p.remote_start, nr = N - rs;
  float thr = 0.0f;
  bool by_ratio = false;
  float mx = 0.0f;
  if (nr > 0) {
    if (p.corr_mode == FFTS_SEL_TOPK) {
      for (int t = threadIdx.x; t < nr; t += blockDim.x) keys[t] = f32_key(corr[FFTS_INDEX(rs + t, N)]);
      __syncthreads();
      const float ranks = __fmul_rn(p.corr_quantile, (float)(nr - 1));
      const int lo = (int)ranks;
      const int hi = (int)ceilf(ranks);
      const float w = __fsub_rn(ranks, (float)lo);
      const float a = key_f32(block_select_rank(keys, nr, lo, hist, bc));
      const float bb = hi == lo ? a : key_f32(block_select_rank(keys, nr, hi, hist, bc));
      const float diff = __fsub_rn(bb, a);
      thr = fabsf(w) < 0.5f ? __fmaf_rn(w, diff, a) : __fmaf_rn(-diff, __fsub_rn(1.0f, w), bb);
    } else {
      float m = -INFINITY;
      for (int t = rs + threadIdx.x; t < N; t += blockDim.x) m = fmaxf(m, corr[FFTS_INDEX(t, N)]);
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      __syncthreads();
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
      __syncthreads();
      if (threadIdx.x == 0) {
        float m2 = red[0];
        for (int w = 1; w < int(blockDim.x >> 5); ++w) m2 = fmaxf(m2, red[w]);
        red[0] = m2;
      }
      __syncthreads();
      mx = red[0] < 1e-6f ? 1e-6f : red[0];
      by_ratio = true;
      thr = p.corr_threshold;
    }
  }
  __syncthreads();
  uint32_t *out = tausel + int64_t(bh) * W;
  for (int w = threadIdx.x; w < W; w += blockDim.x) {
    uint32_t word = 0;
    for (int b = 0; b < 32; ++b) {
      const int t = w * 32 + b;
      if (t >= rs && t < N) {
        const float c = corr[t];
        const bool on = by_ratio ? (__fdiv_rn(c, mx) >= thr) : (c >= thr);
        word |= uint32_t(on) << b;
      }
    }
    out[w] = word;
  }
}

// --------------------------------------------------------- dot products
template <typename T>
__device__ __forceinline__ double dot64_rows(const T *a, const T *b, int D) {
  constexpr int VEC = Elem<T>::kVec;
  double acc = 0.0;
  for (int d = 0; d < D; d += VEC) {
    float av[VEC], bv[VEC];
    load_vec_f32<T>(a + d, av);
    load_vec_f32<T>(b + d, bv);
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc = __fma_rn((double)av[e], (double)bv[e], acc);
  }
  return acc;
}

// 256-lane canonical reduction of per-thread partials (blockDim.x == 256).
__device__ double lane_tree(double v, double *part) {
  part[threadIdx.x] = v;
  __syncthreads();
  for (int s = kLanes / 2; s >= 1; s >>= 1) {
    if (threadIdx.x < s) part[threadIdx.x] = __dadd_rn(part[threadIdx.x], part[threadIdx.x + s]);
    __syncthreads();
  }
  const double r = part[0];
  __syncthreads();
  return r;
}

// ------------------------------------------------------ exact fp32 products
// safe[head][part] = 1 when every pooled value of the head's part (q heads
// first, then k heads; contiguous N x D each, kRangeParts CTAs per head) is zero
// or has a magnitude in [2^-63, 2^64).
// The product of two such bf16 values is exact in fp32: 8 + 8 significant bits
// and a normal exponent.  An fp64 sum that adds (double)(a * b) formed in fp32
// therefore equals the canonical exact-product chain fma((double)a, (double)b,
// acc) bit for bit, with one conversion per term instead of two.  fp32 inputs
// never take this path (their products are not exact in fp32).
constexpr int kRangeParts = 4;  // CTAs per head, each flags its share of the head's values

__global__ void __launch_bounds__(256) exact_range_kernel(const uint4 *__restrict__ qb, const uint4 *__restrict__ kb,
                                                          int64_t nq_heads, int64_t vec_per_head,
                                                          int32_t *__restrict__ safe) {
  const int64_t head = blockIdx.x / kRangeParts;
  const int part = blockIdx.x % kRangeParts;
  const uint4 *src = head < nq_heads ? qb + head * vec_per_head : kb + (head - nq_heads) * vec_per_head;
  int ok = 1;
  for (int64_t i = threadIdx.x + int64_t(part) * blockDim.x; i < vec_per_head; i += int64_t(blockDim.x) * kRangeParts) {
    const uint4 v = src[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t mag = (w[e >> 1] >> (16 * (e & 1))) & 0x7fffu;  // bf16 magnitude bits
      ok &= int(mag == 0u || (mag >= (64u << 7) && mag < (191u << 7)));
    }
  }
  ok = __syncthreads_and(ok);
  if (threadIdx.x == 0) safe[blockIdx.x] = ok;
}

// Every part of the head's values allows exact fp32 products.
__device__ __forceinline__ bool range_ok(const int32_t *__restrict__ safe, int64_t head) {
  bool ok = true;
#pragma unroll
  for (int i = 0; i < kRangeParts; ++i) ok = ok && safe[head * kRangeParts + i] != 0;
  return ok;
}

// ------------------------------------------------------- stripe statistic
// One CTA per (b, h, group of sampled lags whose lags lie within kDiagSpan
// blocks of each other): the normalised variance of the adjacent differences
// along each sampled block-score diagonal (my_attn_v7.py:342-351), written to
// nv[bh * 64 + s]; corr_select_kernel averages them in sample order.  The k rows
// of a tile (128 rows, or 64 where shared memory is short) and the q rows every
// lag of the group pairs them with are staged in shared memory once per tile;
// each score is one fp64 chain in d order, and the three reductions per lag are
// the 256-lane canonical ones.  A thread forms kDiagChains scores of one k row
// (lags g, g + 256 / tile, ...) side by side: the chains' fp64 additions are
// independent, so their latencies overlap, and the k row is read once for all.
constexpr int kDiagTileMax = 128;
constexpr int kDiagTileMin = 64;
constexpr int kDiagChains = 4;
constexpr int kDiagGroup = 8;

// row stride (elements) of staged rows: an odd number of 32-bit words
template <typename T>
__host__ __device__ constexpr int stage_stride(int D) { return D + (sizeof(T) == 2 ? 2 : 1); }

struct DiagGroups {
  int n;                     // groups per (b, h)
  unsigned char first[64];   // first sample index of each group
  unsigned char count[64];   // samples in each group
};

template <typename T>
__device__ void diag_group_body(const T *__restrict__ qb, const T *__restrict__ kb, int H, int Hkv, int D,
                                const ffts_mask_params &p, double *__restrict__ nv, int first, int G, int bh,
                                int gmax, int dt, unsigned char *smem_raw, const int32_t *__restrict__ safe_q,
                                const int32_t *__restrict__ safe_k) {
  const int N = p.n_blocks;
  const int QS = stage_stride<T>(D);
  const int tid = threadIdx.x;
  int lo = p.diag_taus[FFTS_INDEX(first, FFTS_MAX_DIAG_SAMPLES)], hi = lo;
  for (int g = 1; g < G; ++g) {
    lo = min(lo, p.diag_taus[FFTS_INDEX(first + g, FFTS_MAX_DIAG_SAMPLES)]);
    hi = max(hi, p.diag_taus[FFTS_INDEX(first + g, FFTS_MAX_DIAG_SAMPLES)]);
  }
  const int wrows = dt + (hi - lo);
  T *ks = reinterpret_cast<T *>(smem_raw);           // [dt][QS]
  T *qw = ks + dt * QS;                               // [wrows][QS]
  float *vals = reinterpret_cast<float *>(smem_raw + ((size_t(dt + wrows) * QS * sizeof(T) + 15) & ~size_t(15)));
  // [gmax][256], 16-byte aligned whatever gmax * N is
  double *part = reinterpret_cast<double *>((reinterpret_cast<uintptr_t>(vals + gmax * N) + 15) & ~uintptr_t(15));
  const int b = bh / H, h = bh % H;
  const int kh = b * Hkv + h / (H / Hkv);
  const T *q = qb + int64_t(bh) * N * D;
  const T *k = kb + int64_t(kh) * N * D;
  const double sqrtD = sqrt((double)D);
  constexpr int V = Elem<T>::kVec;
  const int vrow = D / V;
  const int mmax = N - lo - 1;
  for (int t0 = 0; t0 < mmax; t0 += dt) {
    // k rows [t0, t0 + dt) and q rows [t0 + lo, t0 + hi + dt)
    constexpr int U = 8;  // 16-byte loads in flight per thread before their stores
    const int total = (dt + wrows) * vrow;
    for (int base = tid; base < total; base += U * blockDim.x) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int idx = base + u * blockDim.x;
        const int rr = idx / vrow, v = idx - rr * vrow;
        const bool isk = rr < dt;
        const int row = isk ? t0 + rr : t0 + lo + (rr - dt);
        if (idx < total && row < N) raw[u] = *reinterpret_cast<const uint4 *>((isk ? k : q) + int64_t(row) * D + v * V);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int idx = base + u * blockDim.x;
        const int rr = idx / vrow, v = idx - rr * vrow;
        const bool isk = rr < dt;
        const int row = isk ? t0 + rr : t0 + lo + (rr - dt);
        if (idx < total && row < N) {
          T *dst = isk ? ks + rr * QS : qw + (rr - dt) * QS;
          const T *e = reinterpret_cast<const T *>(&raw[u]);
#pragma unroll
          for (int c = 0; c < V; ++c) dst[v * V + c] = e[c];
        }
      }
    }
    __syncthreads();
    // kDiagChains scores per thread: (lag g + c * 256 / dt, row t) for c < kDiagChains,
    // all on the k row t (blockDim.x = 256 is a multiple of dt)
    for (int base = tid; base < G * dt; base += kDiagChains * blockDim.x) {
      const int t = t0 + base % dt;  // the same row for every chain of this thread
      int gc[kDiagChains];
      bool vc[kDiagChains];
      const T *qc[kDiagChains];
#pragma unroll
      for (int c = 0; c < kDiagChains; ++c) {
        const int idx = base + c * blockDim.x;
        gc[c] = idx / dt;
        const int tau = p.diag_taus[first + min(gc[c], G - 1)];
        vc[c] = idx < G * dt && t < N - tau - 1;
        // the q row t + tau lies in the staged window [t0 + lo, t0 + hi + dt)
        qc[c] = qw + FFTS_INDEX(t + tau - t0 - lo, wrows) * QS;
      }
      const T *ka = ks + (t - t0) * QS;
      double a[kDiagChains];
#pragma unroll
      for (int c = 0; c < kDiagChains; ++c) a[c] = 0.0;
      bool exact32 = false;
      if constexpr (sizeof(T) == 2) exact32 = safe_q != nullptr && range_ok(safe_q, bh) && range_ok(safe_k, kh);
      if (exact32) {
        for (int d = 0; d < D; ++d) {
          const float kf = Elem<T>::to_f32(ka[d]);
#pragma unroll
          for (int c = 0; c < kDiagChains; ++c)
            a[c] = __dadd_rn(a[c], (double)__fmul_rn(Elem<T>::to_f32(qc[c][d]), kf));
        }
      } else {
        for (int d = 0; d < D; ++d) {
          const double kd = (double)Elem<T>::to_f32(ka[d]);
#pragma unroll
          for (int c = 0; c < kDiagChains; ++c) a[c] = __fma_rn((double)Elem<T>::to_f32(qc[c][d]), kd, a[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < kDiagChains; ++c)
        if (vc[c] && FFTS_IN_RANGE(gc[c], gmax)) vals[gc[c] * N + t] = __double2float_rn(__ddiv_rn(a[c], sqrtD));
    }
    __syncthreads();
  }
  // three canonical reductions per lag, the G lags side by side
  auto tree = [&](double *a) {
#pragma unroll
    for (int g = 0; g < kDiagGroup; ++g)
      if (g < G) part[g * kLanes + tid] = a[g];
    __syncthreads();
    for (int st = kLanes / 2; st >= 1; st >>= 1) {
      for (int idx = tid; idx < G * st; idx += blockDim.x) {
        const int g = idx / st, i = idx - g * st;
        part[g * kLanes + i] = __dadd_rn(part[g * kLanes + i], part[g * kLanes + i + st]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int g = 0; g < kDiagGroup; ++g)
      if (g < G) a[g] = part[g * kLanes];
    __syncthreads();
  };
  double acc[kDiagGroup], mean[kDiagGroup], var[kDiagGroup];
#pragma unroll
  for (int g = 0; g < kDiagGroup; ++g) {
    if (g >= G) break;
    const int n = N - p.diag_taus[first + g] - 2;
    acc[g] = 0.0;
    for (int e = tid; e < n; e += blockDim.x)
      acc[g] = __dadd_rn(acc[g], (double)__fsub_rn(vals[g * N + e + 1], vals[g * N + e]));
  }
  tree(acc);
#pragma unroll
  for (int g = 0; g < kDiagGroup; ++g) {
    if (g >= G) break;
    const int n = N - p.diag_taus[first + g] - 2;
    mean[g] = n >= 2 ? __ddiv_rn(acc[g], (double)n) : 0.0;
    acc[g] = 0.0;
    for (int e = tid; e < n; e += blockDim.x) {
      const double dv = __dsub_rn((double)__fsub_rn(vals[g * N + e + 1], vals[g * N + e]), mean[g]);
      acc[g] = __dadd_rn(acc[g], __dmul_rn(dv, dv));
    }
  }
  tree(acc);
#pragma unroll
  for (int g = 0; g < kDiagGroup; ++g) {
    if (g >= G) break;
    const int n = N - p.diag_taus[first + g] - 2;
    var[g] = n >= 2 ? __ddiv_rn(acc[g], (double)(n - 1)) : __longlong_as_double(0x7ff8000000000000ll);
    const int m = n + 1;
    acc[g] = 0.0;
    for (int e = tid; e < m; e += blockDim.x) acc[g] = __dadd_rn(acc[g], fabs((double)vals[g * N + e]));
  }
  tree(acc);
  if (tid == 0) {
    const double floor6 = (double)1e-6f;
#pragma unroll
    for (int g = 0; g < kDiagGroup; ++g) {
      if (g >= G) break;
      const int m = N - p.diag_taus[first + g] - 1;
      double mabs = m > 0 ? __ddiv_rn(acc[g], (double)m) : __longlong_as_double(0x7ff8000000000000ll);
      if (mabs < floor6) mabs = floor6;
      if (FFTS_IN_RANGE(first + g, FFTS_MAX_DIAG_SAMPLES))
        nv[int64_t(bh) * FFTS_MAX_DIAG_SAMPLES + first + g] = __ddiv_rn(var[g], mabs);
    }
  }
}

// Consecutive sampled lags grouped while their spread stays within the span the
// staged q window covers and the lag values fit in shared memory.
static DiagGroups make_diag_groups(const ffts_mask_params &p, int gmax, int span) {
  DiagGroups gr{};
  int s = 0;
  while (s < p.n_diag_samples) {
    int lo = p.diag_taus[s], hi = lo, c = 1;
    while (s + c < p.n_diag_samples && c < gmax) {
      const int t = p.diag_taus[s + c];
      if (std::max(hi, t) - std::min(lo, t) > span) break;
      lo = std::min(lo, t);
      hi = std::max(hi, t);
      ++c;
    }
    gr.first[gr.n] = (unsigned char)s;
    gr.count[gr.n] = (unsigned char)c;
    ++gr.n;
    s += c;
  }
  return gr;
}

// ------------------------------------------------------------ head stats
// Hot key columns (create_column_block_mask, my_attn_v7.py:403-437) and the last
// query row's top-k (create_last_block_query_mask, :54-72) of one (b, h).
// Column scores are produced whenever the column mask is on; the mask
// composition applies them only where the reference does (stripe heads, or all
// heads without the lag mask).  The q and k rows are staged from row N-1
// downwards in chunks of C rows (16-byte loads, odd-word row strides); the
// suffix sums over q (rows <= N-2, fp64, in row order from N-2 down) are kept
// per channel by D threads and stored per row; then one thread per row forms
// the column score (fp64 FMA chain over d) while another forms the last query
// row's score against the same staged k row.
__host__ __device__ constexpr size_t colrow_smem_for(int C, int N, int D, int elem) {
  return ((2 * size_t(C) * size_t(D + (elem == 2 ? 2 : 1)) * elem + 15) & ~size_t(15)) + size_t(C) * (D + 1) * 8 +
         size_t(D) * 8 + size_t(N) * 8 + size_t((N + 31) / 32) * 4 + 16;
}

// rows per chunk: the largest of 128, 64, 32 whose buffers fit in 200 KB
__host__ __device__ constexpr int colrow_rows(int N, int D, int elem) {
  return colrow_smem_for(128, N, D, elem) <= 200 * 1024 ? 128 : (colrow_smem_for(64, N, D, elem) <= 200 * 1024 ? 64 : 32);
}

static size_t colrow_smem(int N, int D, size_t elem) {
  return colrow_smem_for(colrow_rows(N, D, int(elem)), N, D, int(elem));
}

template <typename T>
__device__ void colrow_body(const T *__restrict__ qb, const T *__restrict__ kb, int H, int Hkv, int D,
                            const ffts_mask_params &p, uint32_t *__restrict__ colsel,
                            uint32_t *__restrict__ lastsel, int bh, unsigned char *smem_raw, int *hist, int *bc) {
  const int N = p.n_blocks;
  const int W = (N + 31) / 32;
  const int C = colrow_rows(N, D, int(sizeof(T)));
  const int QS = stage_stride<T>(D);
  const int PS = D + 1;
  const int tid = threadIdx.x;
  T *qs = reinterpret_cast<T *>(smem_raw);                       // [C][QS]
  T *ks = qs + C * QS;                                            // [C][QS]
  double *pch = reinterpret_cast<double *>(smem_raw + ((2 * size_t(C) * QS * sizeof(T) + 15) & ~size_t(15)));
  double *ql = pch + C * PS;                                      // [D] last q row
  uint32_t *ckeys = reinterpret_cast<uint32_t *>(ql + D);         // [N]
  uint32_t *lkeys = ckeys + N;                                    // [N]
  uint32_t *words = lkeys + N;                                    // [W]
  const int b = bh / H, h = bh % H;
  const T *q = qb + int64_t(bh) * N * D;
  const T *k = kb + (int64_t(b) * Hkv + h / (H / Hkv)) * N * D;
  const double sqrtD = sqrt((double)D);
  const bool col = p.col_on && p.col_end > p.col_start;
  const bool last = p.last_on != 0;
  constexpr int V = Elem<T>::kVec;
  const int vrow = D / V;

  for (int d = tid; d < D; d += blockDim.x) ql[d] = (double)Elem<T>::to_f32(q[int64_t(N - 1) * D + d]);
  double P = 0.0;  // suffix sum of channel tid (tid < D)
  if (col || last) {
    for (int jhi = N - 1; jhi >= 0; jhi -= C) {
      const int rows = min(C, jhi + 1);
      // eight 16-byte loads in flight per thread before their stores
      constexpr int U = 8;
      for (int base = tid; base < 2 * rows * vrow; base += U * blockDim.x) {
        uint4 raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int idx = base + u * blockDim.x;
          if (idx < 2 * rows * vrow) {
            const bool isk = idx >= rows * vrow;
            const int i2 = isk ? idx - rows * vrow : idx;
            const int t = i2 / vrow, v = i2 - t * vrow;
            raw[u] = *reinterpret_cast<const uint4 *>((isk ? k : q) + int64_t(jhi - t) * D + v * V);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int idx = base + u * blockDim.x;
          if (idx < 2 * rows * vrow) {
            const bool isk = idx >= rows * vrow;
            const int i2 = isk ? idx - rows * vrow : idx;
            const int t = i2 / vrow, v = i2 - t * vrow;
            const T *e = reinterpret_cast<const T *>(&raw[u]);
            T *dst = (isk ? ks : qs) + t * QS + v * V;
#pragma unroll
            for (int c = 0; c < V; ++c) dst[c] = e[c];
          }
        }
      }
      __syncthreads();
      if (col && tid < D) {
        // eight rows of channel tid read into registers before their part of the
        // chain: the loads then do not wait behind the previous rows' stores of pch
        // (same shared memory), and the additions keep their order
        for (int t0 = 0; t0 < rows; t0 += 8) {
          double dv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) dv[u] = t0 + u < rows ? (double)Elem<T>::to_f32(qs[(t0 + u) * QS + tid]) : 0.0;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int t = t0 + u;
            if (t < rows) {
              if (jhi - t <= N - 2) P = __dadd_rn(P, dv[u]);
              pch[t * PS + tid] = P;
            }
          }
        }
      }
      __syncthreads();
      // threads [0, C): column scores; threads [C, 2C): last-row scores
      const int t = tid < C ? tid : tid - C;
      if (t < rows && tid < 2 * C) {
        const int j = jhi - t;
        const T *kr = ks + t * QS;
        if (tid < C) {
          if (col) {
            double acc = 0.0;
            for (int d = 0; d < D; ++d) acc = __fma_rn(pch[t * PS + d], (double)Elem<T>::to_f32(kr[d]), acc);
            const int cnt = max(1, N - j - 1);
            ckeys[j] = f32_key(__double2float_rn(__ddiv_rn(__ddiv_rn(acc, sqrtD), (double)cnt)));
          }
        } else if (last) {
          double acc = 0.0;
          for (int d = 0; d < D; ++d) acc = __fma_rn(ql[d], (double)Elem<T>::to_f32(kr[d]), acc);
          lkeys[j] = f32_key(Elem<T>::round_f32(__double2float_rn(acc)));
        }
      }
      __syncthreads();
    }
  }
  for (int w = tid; w < W; w += blockDim.x) words[w] = 0;
  __syncthreads();
  if (col && FFTS_IN_RANGE(p.col_start, N) && FFTS_IN_RANGE(p.col_end - 1, N))
    block_topk_bits(ckeys, p.col_start, p.col_end, p.col_topk, words, hist, bc);
  __syncthreads();
  for (int w = tid; w < W; w += blockDim.x) colsel[int64_t(bh) * W + w] = words[w];
  __syncthreads();
  for (int w = tid; w < W; w += blockDim.x) words[w] = 0;
  __syncthreads();
  if (last) block_topk_bits(lkeys, 0, N, p.last_topk, words, hist, bc);
  __syncthreads();
  for (int w = tid; w < W; w += blockDim.x) lastsel[int64_t(bh) * W + w] = words[w];
}

// Stage 1 of the selection: every independent per-head job of the path in one
// launch, so that these small latency-bound jobs run side by side across the
// SMs.  The longest jobs come first: blocks [0, BH) the column and last-row
// selections (one per (b, h)), the next BH * groups the stripe statistics of
// groups of sampled lags, and the last nF blocks the FFT partial spectra (one
// per (b, h, 8-channel chunk)): the register FFT for R = M / 32 > 0, else the
// shared-memory FFT.
template <typename T, int R>
__global__ void __launch_bounds__(256, 1) select_stage1_kernel(const T *__restrict__ qb, const T *__restrict__ kb,
                                                               int H, int Hkv, int D, ffts_mask_params p, int M,
                                                               int nf, int nchunk, int nBH, int nDG,
                                                               DiagGroups gr, int gmax, int dtile,
                                                               float2 *__restrict__ partial, double *__restrict__ nv,
                                                               uint32_t *__restrict__ colsel,
                                                               uint32_t *__restrict__ lastsel,
                                                               const int32_t *__restrict__ safe_q,
                                                               const int32_t *__restrict__ safe_k) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int hist[256];
  __shared__ int bc[4];
  const int bid = blockIdx.x;
  if (bid < nBH) {
    colrow_body<T>(qb, kb, H, Hkv, D, p, colsel, lastsel, bid, smem_raw, hist, bc);
  } else if (bid < nBH + nDG) {
    const int e = bid - nBH, g = e % gr.n;
    diag_group_body<T>(qb, kb, H, Hkv, D, p, nv, gr.first[g], gr.count[g], e / gr.n, gmax, dtile, smem_raw, safe_q,
                       safe_k);
  } else {
    const int f = bid - nBH - nDG;
    if constexpr (R > 0)
      fft_warp_body<T, R>(qb, kb, H, Hkv, p.n_blocks, D, nchunk, partial, f, smem_raw);
    else
      fft_partial_body<T>(qb, kb, H, Hkv, p.n_blocks, D, M, nf, partial, f % nchunk, nchunk, f / nchunk,
                          smem_raw);
  }
}

// ------------------------------------------------------- warp selection
__device__ uint32_t warp_select_rank(const uint32_t *keys, int n, int rank, int *hist) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0, mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = lane; i < 256; i += 32) hist[i] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const uint32_t kk = keys[i];
      if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 255], 1);
    }
    __syncwarp();
    int c[8], s = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      c[e] = hist[lane * 8 + e];
      s += c[e];
    }
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int excl = incl - s;
    const unsigned ball = __ballot_sync(0xffffffffu, rank >= excl && rank < incl);
    const int src = ball ? __ffs(ball) - 1 : 31;
    int dsel = 255, below = excl;
    if (lane == src) {
      int cc = excl;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (cc + c[e] > rank) { dsel = lane * 8 + e; below = cc; break; }
        cc += c[e];
      }
    }
    dsel = __shfl_sync(0xffffffffu, dsel, src);
    below = __shfl_sync(0xffffffffu, below, src);
    rank -= below;
    prefix |= uint32_t(dsel) << shift;
    mask |= 0xffu << shift;
    __syncwarp();
  }
  return prefix;
}

// k largest of keys[0..n) (ties: lowest index) OR-ed into words[] (warp-local).
__device__ void warp_topk_bits(const uint32_t *keys, int n, int k, uint32_t *words, int *hist) {
  const int lane = threadIdx.x & 31;
  if (k >= n) {
    for (int j = lane; j < n; j += 32) atomicOr(&words[j >> 5], 1u << (j & 31));
    __syncwarp();
    return;
  }
  const uint32_t T = warp_select_rank(keys, n, n - k, hist);
  int gt = 0;
  for (int j = lane; j < n; j += 32) gt += keys[j] > T;
  for (int o = 16; o; o >>= 1) gt += __shfl_xor_sync(0xffffffffu, gt, o);
  const int need = k - gt;
  int base = 0;
  for (int c = 0; c < n; c += 32) {
    const int j = c + lane;
    const bool in = j < n;
    const uint32_t kk = in ? keys[j] : 0u;
    const bool eq = in && kk == T;
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    const int before = base + __popc(bal & ((1u << lane) - 1));
    if (in && (kk > T || (eq && before < need))) atomicOr(&words[j >> 5], 1u << (j & 31));
    base += __popc(bal);
  }
  __syncwarp();
}

// ------------------------------------------------------------ mask build
// bits t < x of a word (x clipped to [0, 32])
__device__ __forceinline__ uint32_t bits_below(int x) {
  return x <= 0 ? 0u : (x >= 32 ? 0xffffffffu : ((1u << x) - 1u));
}

// bits [base, base + 32) of the bit array words[0..W) as one word (bit k = bit
// base + k); positions outside the array (base may be negative) read as 0
__device__ __forceinline__ uint32_t lag_window(const uint32_t *words, int W, int base) {
  const int wlo = base >> 5, sh = base & 31;  // floor division, also for base < 0
  const uint32_t a = (wlo >= 0 && wlo < W) ? words[FFTS_INDEX(wlo, W)] : 0u;
  const uint32_t b = (wlo + 1 >= 0 && wlo + 1 < W) ? words[FFTS_INDEX(wlo + 1, W)] : 0u;
  return sh ? (a >> sh) | (b << (32 - sh)) : a;
}

template <typename T>
__global__ void __launch_bounds__(256) mask_build_kernel(const T *__restrict__ qb,
                                                         const T *__restrict__ kb, int H, int Hkv,
                                                         int D, ffts_mask_params p, int R,
                                                         const int32_t *__restrict__ stripe_ws,
                                                         const uint32_t *__restrict__ tausel,
                                                         const uint32_t *__restrict__ colsel,
                                                         const uint32_t *__restrict__ lastsel,
                                                         uint32_t *__restrict__ bits,
                                                         int32_t *__restrict__ row_count) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int VEC = Elem<T>::kVec;
  constexpr int RMAX = 16;
  const int N = p.n_blocks;
  const int W = (N + 31) / 32;
  double *qrow = reinterpret_cast<double *>(smem_raw);        // [R][D]
  uint32_t *keys = reinterpret_cast<uint32_t *>(qrow + R * D);  // [R][N]
  uint32_t *rowbits = keys + R * N;                           // [R][W]
  int *hist = reinterpret_cast<int *>(rowbits + R * W);       // [8][256]
  int *cnt = hist + 8 * 256;                                  // [R]
  const int bh = blockIdx.y;
  const int i0 = blockIdx.x * R;
  const int rows = min(R, N - i0);
  const int b = bh / H, h = bh % H;
  const int stripe = stripe_ws[bh];
  const bool diffuse = p.corr_on && !stripe;
  const int col_apply = p.col_on && (!p.corr_on || stripe);
  for (int e = threadIdx.x; e < R * W; e += blockDim.x) rowbits[e] = 0;
  for (int e = threadIdx.x; e < R; e += blockDim.x) cnt[e] = 0;

  if (diffuse) {
    const T *q = qb + int64_t(bh) * N * D;
    const T *k = kb + (int64_t(b) * Hkv + h / (H / Hkv)) * N * D;
    for (int e = threadIdx.x; e < rows * D; e += blockDim.x)
      qrow[e] = (double)Elem<T>::to_f32(q[int64_t(i0) * D + e]);
    __syncthreads();
    const double sqrtD = sqrt((double)D);
    const int jmax = i0 + rows;  // columns 0 .. i0+rows-1
    for (int j = threadIdx.x; j < jmax; j += blockDim.x) {
      double acc[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) acc[r] = 0.0;
      const T *kr = k + int64_t(j) * D;
      for (int d = 0; d < D; d += VEC) {
        float kv[VEC];
        load_vec_f32<T>(kr + d, kv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const double kd = (double)kv[e];
#pragma unroll
          for (int r = 0; r < RMAX; ++r)
            if (r < rows) acc[r] = __fma_rn(qrow[r * D + d + e], kd, acc[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        if (r < rows) keys[r * N + j] = f32_key(__double2float_rn(__ddiv_rn(acc[r], sqrtD)));
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    for (int r = warp; r < rows; r += blockDim.x >> 5) {
      const int i = i0 + r;
      const float kf = __fmul_rn((float)(i + 1), p.qk_topk_ratio);
      int ki = (int)kf;
      if (ki < 1) ki = 1;
      warp_topk_bits(keys + r * N, i + 1, ki, rowbits + r * W, hist + warp * 256);
    }
  }
  __syncthreads();

  const uint32_t *ts = tausel + int64_t(bh) * W;
  const uint32_t *cs = colsel + int64_t(bh) * W;
  const uint32_t *ls = lastsel + int64_t(bh) * W;
  const bool lag_on = p.corr_on && stripe;
  for (int e = threadIdx.x; e < rows * W; e += blockDim.x) {
    const int r = e / W, w = e - r * W;
    const int i = i0 + r;
    const int j0 = w * 32;  // bit t of the word is key block j = j0 + t, lag tau = i - j
    // kept: j < keep_sink, j >= N - keep_recent, tau <= local_window (j >= i - local_window),
    // and for a stripe head with the lag mask the selected lags tau >= remote_start
    // (j <= i - remote_start) among j >= keep_sink; then the diffuse, column and
    // last-row selections; nothing above the diagonal (j <= i)
    uint32_t word = bits_below(p.keep_sink - j0) | ~bits_below(N - p.keep_recent - j0) |
                    ~bits_below(i - p.local_window - j0);
    if (lag_on) {
      // bit t <- selected-lag bit tau = i - j0 - t: the 32 lag bits from tau = i - j0 - 31
      // up, reversed
      const uint32_t lagw = __brev(lag_window(ts, W, i - j0 - 31));
      word |= lagw & bits_below(i - p.remote_start + 1 - j0) & ~bits_below(p.keep_sink - j0);
    }
    if (diffuse) word |= rowbits[r * W + w];
    if (col_apply) word |= cs[w];
    if (p.last_on && i == N - 1) word |= ls[w];
    word &= bits_below(i + 1 - j0);
    bits[(int64_t(bh) * N + i) * W + w] = word;
    atomicAdd(&cnt[r], __popc(word));
  }
  __syncthreads();
  if (row_count)
    for (int r = threadIdx.x; r < rows; r += blockDim.x) row_count[int64_t(bh) * N + i0 + r] = cnt[r];
}

__global__ void unpack_kernel(const uint32_t *__restrict__ bits, int64_t rows, int64_t N,
                              uint8_t *__restrict__ out) {
  const int64_t W = (N + 31) / 32;
  const int64_t total = rows * N;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / N, j = e - r * N;
    out[e] = (bits[r * W + (j >> 5)] >> (j & 31)) & 1u;
  }
}

// ------------------------------------------------------------- host side
struct MaskWorkspace {
  float2 *partial;
  double *nv;  // [B*H][FFTS_MAX_DIAG_SAMPLES] per-lag stripe statistics
  uint32_t *tausel, *colsel, *lastsel;
  int32_t *stripe;
  int32_t *safe;  // [B*H q heads, then up to B*H k heads][kRangeParts]: exact fp32 products (exact_range_kernel)
  int64_t bytes;
};

static inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

static MaskWorkspace carve(void *ws, int64_t B, int64_t H, int64_t N, int64_t D) {
  MaskWorkspace m{};
  const int M = 1 << ilog2_ceil(2 * N);
  const int64_t F = M / 2 + 1;
  const int64_t nchunk = ceil_div(D, kDChunk);
  const int64_t W = ceil_div(N, 32);
  char *p = static_cast<char *>(ws);
  int64_t off = 0;
  m.partial = reinterpret_cast<float2 *>(p + off);
  off += align256(B * H * nchunk * F * int64_t(sizeof(float2)));
  m.nv = reinterpret_cast<double *>(p + off);
  off += align256(B * H * FFTS_MAX_DIAG_SAMPLES * 8);
  m.tausel = reinterpret_cast<uint32_t *>(p + off);
  off += align256(B * H * W * 4);
  m.colsel = reinterpret_cast<uint32_t *>(p + off);
  off += align256(B * H * W * 4);
  m.lastsel = reinterpret_cast<uint32_t *>(p + off);
  off += align256(B * H * W * 4);
  m.stripe = reinterpret_cast<int32_t *>(p + off);
  off += align256(B * H * 4);
  m.safe = reinterpret_cast<int32_t *>(p + off);
  off += align256(2 * B * H * 4 * kRangeParts);
  m.bytes = off;
  return m;
}

int64_t mask_workspace_bytes(int64_t B, int64_t H, int64_t N, int64_t D) {
  return carve(nullptr, B, H, N, D).bytes;
}

template <typename T>
static int run_block_mask(const T *qb, const T *kb, int64_t B, int64_t H, int64_t Hkv, int64_t D,
                          const ffts_mask_params &p, uint32_t *bits, int32_t *row_count, float *corr,
                          float *csum, uint8_t *is_stripe, float *svar, const MaskWorkspace &ws,
                          cudaStream_t stream) {
  const int N = p.n_blocks;
  const int M = 1 << ilog2_ceil(2 * int64_t(N));
  const int nchunk = int(ceil_div(D, kDChunk));
  const int W = int(ceil_div(N, 32));
  const unsigned BH = unsigned(B * H);
  // which heads' pooled values allow exact fp32 products (bf16 only)
  const int32_t *safe_q = nullptr, *safe_k = nullptr;
  if (sizeof(T) == 2 && D % 8 == 0) {
    const int64_t nq = B * H, nk = B * Hkv;
    exact_range_kernel<<<unsigned((nq + nk) * kRangeParts), 256, 0, stream>>>(reinterpret_cast<const uint4 *>(qb),
                                                             reinterpret_cast<const uint4 *>(kb), nq,
                                                             int64_t(N) * D / 8, ws.safe);
    FFTS_CUDA(cudaGetLastError());
    safe_q = ws.safe;
    safe_k = ws.safe + nq * kRangeParts;
  }
  // stage 1: FFT partial spectra, per-lag stripe statistics, column and last-row selections
  int nf = kDChunk;
  while (nf > 1 && fft_partial_smem(M, nf) > 64 * 1024) nf >>= 1;
  const size_t elem = sizeof(T);
  const int R = (M >= 32 && M <= 2048) ? M / 32 : 0;  // register FFT up to 2048 points
  const int nF = p.corr_on ? nchunk * int(BH) : 0;
  const int gmax = std::max(1, std::min(kDiagGroup, 8192 / N));
  const size_t st = size_t(D + (elem == 2 ? 2 : 1)) * elem;
  const int64_t room = int64_t(200 * 1024) - int64_t(gmax) * N * 4 - int64_t(gmax) * kLanes * 8 - 64;
  // stripe tiles of 128 k rows where the staged rows fit, else 64; lag span up to 192 blocks (64 for fp32)
  const int span_cap = elem == 2 ? 192 : 64;
  const int dtile = room / int64_t(st) - 2 * kDiagTileMax >= span_cap ? kDiagTileMax : kDiagTileMin;
  const int span = int(std::max<int64_t>(0, std::min<int64_t>(span_cap, room / int64_t(st) - 2 * dtile)));
  const DiagGroups gr = make_diag_groups(p, gmax, span);
  const int nDG = (p.corr_on && !p.stripe_all_diffuse) ? gr.n * int(BH) : 0;
  size_t smem1 = colrow_smem(N, int(D), elem);
  if (nDG) smem1 = std::max(smem1, size_t(2 * dtile + span) * st + size_t(gmax) * N * 4 + size_t(gmax) * kLanes * 8 + 64);
  if (nF) smem1 = std::max(smem1, R ? fft_warp_smem_rt(R, N, elem) : fft_partial_smem(M, nf));
  const unsigned grid1 = unsigned(nF + nDG + int(BH));
#define FFTS_STAGE1(RR)                                                                                          \
  case RR: {                                                                                                     \
    {                                                                                                            \
      const int rc1 = ensure_func_smem(reinterpret_cast<const void *>(&select_stage1_kernel<T, RR>), int(smem1)); \
      if (rc1) return rc1;                                                                                       \
    }                                                                                                            \
    select_stage1_kernel<T, RR><<<grid1, 256, smem1, stream>>>(qb, kb, int(H), int(Hkv), int(D), p, M, nf, nchunk, \
                                                               int(BH), nDG, gr, gmax, dtile, ws.partial, ws.nv,  \
                                                               ws.colsel, ws.lastsel, safe_q, safe_k);           \
    break;                                                                                                       \
  }
  switch (R) {
    FFTS_STAGE1(0)
    FFTS_STAGE1(1)
    FFTS_STAGE1(2)
    FFTS_STAGE1(4)
    FFTS_STAGE1(8)
    FFTS_STAGE1(16)
    FFTS_STAGE1(32)
    FFTS_STAGE1(64)
    default:
      set_error(FFTS_E_INVALID, "selection: unsupported FFT length %d", M);
      return FFTS_E_INVALID;
  }
#undef FFTS_STAGE1
  FFTS_CUDA(cudaGetLastError());
  // stage 2: stripe decision, inverse FFT, lag selection
  const size_t smem2 = size_t(M / 2 + M) * sizeof(float2) + size_t(N) * 8;
  {
    const int rc2 = ensure_func_smem(reinterpret_cast<const void *>(&corr_select_kernel), int(smem2));
    if (rc2) return rc2;
  }
  corr_select_kernel<<<BH, 512, smem2, stream>>>(ws.partial, nchunk, N, M, p, ws.nv, ws.stripe, is_stripe, svar,
                                                 corr, csum, ws.tausel);
  FFTS_CUDA(cudaGetLastError());
  const int RT = N <= 1024 ? 16 : max(1, 16384 / N);  // mask rows per CTA
  const size_t smem4 = size_t(RT) * D * 8 + size_t(RT) * N * 4 + size_t(RT) * W * 4 + 8 * 256 * 4 + size_t(RT) * 4;
  {
    const int rc4 = ensure_func_smem(reinterpret_cast<const void *>(&mask_build_kernel<T>), int(smem4));
    if (rc4) return rc4;
  }
  mask_build_kernel<T><<<dim3(unsigned(ceil_div(N, RT)), BH), 256, smem4, stream>>>(
      qb, kb, int(H), int(Hkv), int(D), p, RT, ws.stripe, ws.tausel, ws.colsel, ws.lastsel, bits, row_count);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

int validate_params(const ffts_mask_params &p, int64_t D) {
  const int N = p.n_blocks;
  FFTS_REQUIRE(N >= 1 && N <= kMaxBlocks, "n_blocks %d outside [1, %d]", N, kMaxBlocks);
  FFTS_REQUIRE(!p.corr_on || N >= 10, "the correlation mask needs at least 10 blocks (got %d)", N);
  FFTS_REQUIRE(p.n_diag_samples >= 0 && p.n_diag_samples <= FFTS_MAX_DIAG_SAMPLES, "bad n_diag_samples");
  for (int s = 0; s < p.n_diag_samples; ++s)
    FFTS_REQUIRE(p.diag_taus[s] >= 0 && p.diag_taus[s] < N, "sampled lag %d outside [0, N)", p.diag_taus[s]);
  FFTS_REQUIRE(!p.corr_on || p.stripe_all_diffuse || p.n_diag_samples >= 1, "no sampled diagonals");
  FFTS_REQUIRE(!p.corr_on || (p.remote_start >= 1 && p.remote_start < N), "remote_start outside [1, N)");
  FFTS_REQUIRE(p.exclude_tau >= 0, "exclude_tau < 0");
  FFTS_REQUIRE(p.corr_mode == FFTS_SEL_TOPK || p.corr_mode == FFTS_SEL_THRESHOLD, "bad corr_mode");
  FFTS_REQUIRE(!p.col_on || p.col_end <= p.col_start || (p.col_start >= 0 && p.col_end <= N && p.col_topk >= 1),
               "bad column range");
  FFTS_REQUIRE(!p.last_on || (p.last_topk >= 1 && p.last_topk <= N), "bad last_topk");
  FFTS_REQUIRE(D >= 8 && D <= 256 && D % 8 == 0, "head_dim %lld unsupported for selection", (long long)D);
  return FFTS_OK;
}

int block_mask(const void *qb, const void *kb, int dtype, int64_t B, int64_t H, int64_t Hkv, int64_t D,
               const ffts_mask_params *params, uint32_t *bits, int32_t *row_count, float *corr,
               float *csum, uint8_t *is_stripe, float *svar, void *workspace, int64_t ws_bytes,
               cudaStream_t stream) {
  FFTS_REQUIRE(params != nullptr, "params is NULL");
  const ffts_mask_params &p = *params;
  int rc = validate_params(p, D);
  if (rc) return rc;
  FFTS_REQUIRE(dtype == FFTS_DTYPE_F32 || dtype == FFTS_DTYPE_BF16, "unsupported dtype %d", dtype);
  FFTS_REQUIRE(B >= 1 && H >= 1 && Hkv >= 1 && H % Hkv == 0, "bad head counts H=%lld Hkv=%lld",
               (long long)H, (long long)Hkv);
  FFTS_REQUIRE(B * H <= 65535, "B*H too large");
  FFTS_REQUIRE(qb && kb && bits, "NULL tensor pointer");
  FFTS_REQUIRE((reinterpret_cast<uintptr_t>(qb) & 15) == 0 && (reinterpret_cast<uintptr_t>(kb) & 15) == 0,
               "pooled inputs must be 16-byte aligned");
  const int64_t need = mask_workspace_bytes(B, H, p.n_blocks, D);
  if (workspace == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    set_error(FFTS_E_WORKSPACE, "workspace needs %lld bytes, 256-byte aligned (got %lld)", (long long)need,
              (long long)ws_bytes);
    return FFTS_E_WORKSPACE;
  }
  rc = ensure_tables();
  if (rc) return rc;
  const MaskWorkspace ws = carve(workspace, B, H, p.n_blocks, D);
  if (dtype == FFTS_DTYPE_BF16)
    return run_block_mask(static_cast<const __nv_bfloat16 *>(qb), static_cast<const __nv_bfloat16 *>(kb), B, H,
                          Hkv, D, p, bits, row_count, corr, csum, is_stripe, svar, ws, stream);
  return run_block_mask(static_cast<const float *>(qb), static_cast<const float *>(kb), B, H, Hkv, D, p, bits,
                        row_count, corr, csum, is_stripe, svar, ws, stream);
}

int unpack_mask(const uint32_t *bits, int64_t B, int64_t H, int64_t N, uint8_t *out, cudaStream_t stream) {
  FFTS_REQUIRE(bits && out && B > 0 && H > 0 && N > 0, "bad unpack arguments");
  const int64_t total = B * H * N * N;
  int sms = 1;
  const int rc = device_sm_count(&sms);
  if (rc) return rc;
  // a grid-stride loop: enough CTAs to fill every SM 16 deep, fewer for small masks
  const int blocks = int(std::min<int64_t>(ceil_div(total, 256), int64_t(sms) * 16));
  unpack_kernel<<<blocks, 256, 0, stream>>>(bits, B * H * N, N, out);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
