// qkv_proj.cu -- the caller's QKV projection GEMM with RoPE, the head-major
// layout and the q/k block pooling in its epilogue (tcgen05 + TMEM + TMA).
//
// The caller of myattn_prefill (eval/LongBench/pred.py:177-194 through the HF
// attention forward) projects the hidden states, q/k/v = x W^T (+ bias), views
// them head-major, applies apply_rotary_pos_emb in bf16, and myattn_prefill
// pools the rotated q and k (block_mean_pool, attn_src/fft_attn/my_attn_v7.py:
// 105-114, used at :554-555).  rope_pool.cu does the last three in one pass over
// the projection; this kernel folds them into the projection GEMM itself, so the
// projection never reaches HBM:
//
//   out[t, c] = bf16(sum_k x[t, k] * W[c, k] (+ bias[c]))      fp32 accumulation
//   q, k      = RoPE(out) per head, head-major [B, H, L, 128]  (rope_pool's arithmetic)
//   v         = out per head, head-major
//   pooled    = fp32 sum of a block's rotated bf16 rows in row order from +0,
//               / block_size, rounded to bf16                  (pool_kernel's arithmetic)
//
// W is the caller's q_proj, k_proj and v_proj weights stacked row-wise
// ([(Hq + 2 Hkv) * 128, hidden], torch Linear layout, K-major); head g of the
// product is q head g for g < Hq, then the k heads, then the v heads.
//
// One CTA per SM, persistent over 256 x 256 output tiles (256 tokens x 2 heads):
//   warp 0      TMA producer: x [256 x 64] and W [256 x 64] bf16 per stage into a
//               three-stage ring (SWIZZLE_128B, no multicast).
//   warp 1      MMA issuer (one thread): two M = 128, N = 256 accumulators (the
//               tile's two row halves) fill all 512 TMEM columns; per 64-wide K
//               step 8 tcgen05.mma read the stage, then a commit frees it.
//   warps 2-9   epilogue, four warps per row half (thread = TMEM lane = row): read
//               the accumulator, round it to bf16 in registers (bias added in fp32
//               first) and release TMEM at once, so the next tile's MMAs overlap
//               the rest.  Per head and 64-channel box: RoPE against the cos/sin
//               rows (re-laid first by rope_tile_kernel so that a warp's 32 rows
//               load a chunk in one coalesced access) into a shared-memory box in the TMA SWIZZLE_128B layout, one
//               TMA tensor store of the box into the head-major output (rows past
//               L dropped by the map), and the pooling, one thread per channel
//               summing the box's rows of a block in order.
// A 256 x 256 tile loads 64 KB per 2 x 128 MMA cycles of each K step, 64 B per
// SM clock from L2; a 128-row tile would need 96.  Every mbarrier wait is
// bounded: on a time-out the CTA records a status code, stops, waits (bounded)
// for its own copies and MMAs and frees TMEM.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "ffts_common.cuh"
#include "tc_sm100.cuh"

namespace ffts {
namespace qkv {

using namespace ::ffts::tc;

constexpr int kD = 128;            // head_dim
constexpr int kBM = 256;           // tokens per tile (two M = 128 accumulators)
constexpr int kBN = 256;           // projection columns per tile (two heads)
constexpr int kBK = 64;            // K per stage: one 128-byte swizzle row
constexpr int kStages = 3;
constexpr int kABytes = kBM * kBK * 2;       // 32 KB
constexpr int kBBytes = kBN * kBK * 2;       // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 320;
constexpr int kEpiThreads = 256;
constexpr int kBoxBytes = 128 * 128;  // one staged output box: 128 rows x 64 bf16 (TMA SWIZZLE_128B)
constexpr int kTmemCols = 512;
constexpr double kWaitSeconds = 2.0;
constexpr double kDrainSeconds = 4.0;

// status codes (shared with the attention kernel's word, distinct values)
constexpr int kErrTimeoutProducer = 6;
constexpr int kErrTimeoutMma = 7;
constexpr int kErrTimeoutEpilogue = 8;
constexpr int kErrSmemAlign = 9;

struct Smem {
  static constexpr int stages = 0;
  static constexpr int stage = kStages * kStageBytes;        // one output box per row half
  static constexpr int bars = stage + 2 * kBoxBytes;
  static constexpr int nbars = 2 * kStages + 3;
  static constexpr int tmem_slot = bars + nbars * 8;
  static constexpr int abort = tmem_slot + 4;
  static constexpr int bytes = abort + 12;
};
static_assert(Smem::bytes <= 232448, "exceeds the 227 KB of shared memory a CTA may use");

constexpr int BF = 0;              // stage full   [kStages]
constexpr int BE = BF + kStages;   // stage empty  [kStages]
constexpr int BAF = BE + kStages;  // accumulators complete
constexpr int BAE = BAF + 1;       // accumulators read out (kEpiThreads arrivals)
constexpr int BDR = BAE + 1;       // drain

struct Params {
  const __nv_bfloat16 *bias;  // [heads * 128] or NULL
  __nv_bfloat16 *pooled[2];   // [B, Hq, N, D], [B, Hkv, N, D]
  __nv_bfloat16 *raw;         // optional [B, L, raw_ld] projection before RoPE
  int64_t raw_ld;
  const uint4 *rope;          // cos / sin re-laid by rope_tile_kernel (rope_tile_index)
  int L, N, Hq, Hkv, heads, bs;
  int kblocks;                // K steps of kBK
  int m_tiles, n_tiles, tiles;
  int *status;
  long long wait_cycles, drain_cycles;
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 pr = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&pr);
}

__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// AND of pred over the 128 threads of one row half (named barrier 1 + half).
__device__ __forceinline__ bool half_all(int half, bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(int(pred)), "r"(1 + half)
      : "memory");
  return r != 0;
}

// Barrier of the 128 threads of one row half (named barrier 3 + half).
__device__ __forceinline__ void half_sync(int half) {
  asm volatile("bar.sync %0, 128;" ::"r"(3 + half) : "memory");
}

struct TileCoord {
  int b, mt, nt;
};

__device__ __forceinline__ TileCoord tile_coord(const Params &p, int t) {
  // projection columns fastest: the CTAs resident at one time share a few
  // token blocks of x, and W stays in L2
  TileCoord c;
  c.nt = t % p.n_tiles;
  const int m = t / p.n_tiles;
  c.mt = m % p.m_tiles;
  c.b = m / p.m_tiles;
  return c;
}

// The cos / sin tables re-laid so that the 32 rows of a warp read a 16-byte
// chunk with one coalesced 512-byte access: uint4 [row / 32][16 chunks][cos, sin][row % 32],
// rows past L zero.  (The caller's [L, 128] tables, read by row-per-thread lanes,
// put 32 different rows in every load instruction.)
__host__ __device__ __forceinline__ int64_t rope_tile_index(int64_t row, int chunk, int table) {
  return (((row >> 5) * 16 + chunk) * 2 + table) * 32 + (row & 31);
}

__global__ void __launch_bounds__(256) rope_tile_kernel(const __nv_bfloat16 *__restrict__ cos,
                                                        const __nv_bfloat16 *__restrict__ sin, int64_t cs_ld,
                                                        int64_t L, int64_t rows, uint4 *__restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // output uint4 index
  if (i >= rows * 32) return;
  const int64_t row = (i >> 10) * 32 + (i & 31);
  const int table = int((i >> 5) & 1), chunk = int((i >> 6) & 15);
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (row < L) v = *reinterpret_cast<const uint4 *>((table ? sin : cos) + row * cs_ld + chunk * 8);
  out[i] = v;
}

__global__ void __launch_bounds__(kThreads, 1)
    qkv_rope_pool_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kErrSmemAlign);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return sbase + uint32_t(Smem::bars) + 8u * uint32_t(i); };
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + Smem::abort);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Smem::tmem_slot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(BF + s), 1);
      mbar_init(bar(BE + s), 1);
    }
    mbar_init(bar(BAF), 1);
    mbar_init(bar(BAE), kEpiThreads);
    mbar_init(bar(BDR), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == 0 && lane == 0) {
    prefetch_map(&tm_x);
    prefetch_map(&tm_w);
    prefetch_map(&tm_q);
    prefetch_map(&tm_k);
    prefetch_map(&tm_v);
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const TileCoord c = tile_coord(p, t);
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(bar(BE + s), ((it / kStages) & 1) ^ 1, abort_flag, p.wait_cycles)) {
            ok = false;
            break;
          }
          mbar_arrive_tx(bar(BF + s), kStageBytes);
          const uint32_t dst = sbase + uint32_t(s * kStageBytes);
          tma_load_4d(dst, &tm_x, bar(BF + s), kb * kBK, c.mt * kBM, c.b, 0);
          tma_load_4d(dst + kABytes, &tm_w, bar(BF + s), kb * kBK, c.nt * kBN, 0, 0);
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicCAS(p.status, 0, kErrTimeoutProducer);
        // wait (bounded, ignoring the abort flag) for the copies still in flight
        volatile int never = 0;
        for (int n = max(0, it - kStages); n < it; ++n)
          mbar_wait(bar(BF + n % kStages), (n / kStages) & 1, &never, p.drain_cycles);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(false, kBN);
      // K-major SWIZZLE_128B operands; a 16-element K step is +32 bytes inside the
      // swizzle row, the second row half of x starts 128 rows (16 KB) in
      const uint64_t d0 = smem_desc(sbase, 16, 1024);
      int it = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++i) {
        if (!mbar_wait(bar(BAE), (i & 1) ^ 1, abort_flag, p.wait_cycles)) {
          ok = false;
          break;
        }
        fence_after();
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(bar(BF + s), (it / kStages) & 1, abort_flag, p.wait_cycles)) {
            ok = false;
            break;
          }
          fence_after();
          const uint64_t da = d0 + uint64_t((s * kStageBytes) >> 4);
          const uint64_t db = da + uint64_t(kABytes >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            umma_f16(tmem, da + uint64_t(2 * kk), db + uint64_t(2 * kk), idesc, acc);
            umma_f16(tmem + 256, da + uint64_t((16384 >> 4) + 2 * kk), db + uint64_t(2 * kk), idesc, acc);
          }
          umma_commit(bar(BE + s));
        }
        if (ok) umma_commit(bar(BAF));
      }
      if (!ok) {
        *abort_flag = 1;
        atomicCAS(p.status, 0, kErrTimeoutMma);
      }
      umma_commit(bar(BDR));
      volatile int never = 0;
      mbar_wait(bar(BDR), 0, &never, p.drain_cycles);
    }
  } else {
    // ================================================================ epilogue (warps 2-9)
    const int half = (warp - 2) >> 2;      // row half of the tile
    const int quarter = warp & 3;          // TMEM lanes this warp may access: 32 * (warp % 4) + [0, 32)
    const int r = quarter * 32 + lane;     // row within the half == TMEM lane
    const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(half * 256);
    uint8_t *stage = smem + Smem::stage + half * kBoxBytes;  // this half's staged output box
    const uint32_t stage_s = sbase + uint32_t(Smem::stage + half * kBoxBytes);
    const float fbs = float(p.bs);
    bool ok = true;
    int i = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++i) {
      const TileCoord c = tile_coord(p, t);
      if (!half_all(half, mbar_wait(bar(BAF), i & 1, abort_flag, p.wait_cycles))) {
        ok = false;
        break;
      }
      fence_after();
      // ---- accumulator -> bf16 pairs in registers (+ bias in fp32), then TMEM is free
      uint32_t pk[128];
      const int col0 = c.nt * kBN;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        float f[32];
        tmem_ld32(taddr + uint32_t(cc * 32), f);
        tmem_wait_ld();
        if (p.bias != nullptr && col0 + cc * 32 < p.heads * kD) {
          const uint4 *bp = reinterpret_cast<const uint4 *>(p.bias + col0 + cc * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 bw = __ldg(bp + q4);
            const uint32_t w4[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              f[q4 * 8 + 2 * e] = __fadd_rn(f[q4 * 8 + 2 * e], lo_f(w4[e]));
              f[q4 * 8 + 2 * e + 1] = __fadd_rn(f[q4 * 8 + 2 * e + 1], hi_f(w4[e]));
            }
          }
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[cc * 16 + e] = pack2(f[2 * e], f[2 * e + 1]);
      }
      fence_before();
      mbar_arrive(bar(BAE));

      const int t_half = c.mt * kBM + half * 128;  // first token of this row half
      const int tl = t_half + r;                     // this thread's token within the sequence
      const bool valid = tl < p.L;
      if (p.raw != nullptr && valid) {
        __nv_bfloat16 *dst = p.raw + (int64_t(c.b) * p.L + tl) * p.raw_ld + col0;
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if (col0 + q * 8 < p.heads * kD)
            *reinterpret_cast<uint4 *>(dst + q * 8) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      if (t_half >= p.L) continue;  // a row half wholly past the sequence (uniform over the half)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int g = c.nt * 2 + hh;  // head of the stacked projection (uniform over the CTA)
        if (g >= p.heads) break;
        const int role = g < p.Hq ? 0 : (g < p.Hq + p.Hkv ? 1 : 2);
        const int hr = role == 0 ? g : (role == 1 ? g - p.Hq : g - p.Hq - p.Hkv);
        const int hcount = role == 0 ? p.Hq : p.Hkv;
        const CUtensorMap *omap = role == 0 ? &tm_q : (role == 1 ? &tm_k : &tm_v);
        const uint4 *rope = p.rope + rope_tile_index(tl, 0, 0);  // this row's chunk 0 of cos
#pragma unroll
        for (int box = 0; box < 2; ++box) {
          // ---- this row's 64 channels [64 box, 64 box + 64), rotated for q / k, into
          // the staged box: 16-byte chunk c8 of row r at r * 128 + ((c8 ^ (r % 8)) * 16),
          // the TMA SWIZZLE_128B layout (row-per-thread writes and the pooling's
          // column reads are both free of bank conflicts)
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            uint32_t ow[4];
            const int wo = 64 * hh + 32 * box + 4 * c8;        // own words (channels 64 box + 8 c8 ..)
            const int wp = 64 * hh + 32 * (1 - box) + 4 * c8;  // RoPE partners (channels -+ 64)
            if (!valid) {
#pragma unroll
              for (int e = 0; e < 4; ++e) ow[e] = 0u;  // rows past L pool as +0 and are not stored
            } else if (role == 2) {
#pragma unroll
              for (int e = 0; e < 4; ++e) ow[e] = pk[wo + e];
            } else {
              const uint4 cv = rope[(8 * box + c8) * 64];       // cos, channels 64 box + 8 c8 ..
              const uint4 sv = rope[(8 * box + c8) * 64 + 32];  // sin
              const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float o[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  const float x = u ? hi_f(pk[wo + e]) : lo_f(pk[wo + e]);
                  const float xp = u ? hi_f(pk[wp + e]) : lo_f(pk[wp + e]);
                  const float cf = u ? hi_f(cw[e]) : lo_f(cw[e]), sf = u ? hi_f(sw[e]) : lo_f(sw[e]);
                  // rotate_half: -x[d + 64] for d < 64, x[d - 64] for d >= 64
                  o[u] = __fadd_rn(bf(__fmul_rn(x, cf)), bf(__fmul_rn(box ? xp : -xp, sf)));
                }
                ow[e] = pack2(o[0], o[1]);
              }
            }
            *reinterpret_cast<uint4 *>(stage + r * 128 + ((c8 ^ (r & 7)) << 4)) =
                make_uint4(ow[0], ow[1], ow[2], ow[3]);
          }
          fence_proxy_async();
          half_sync(half);
          // one thread stores the box: rows past L fall outside the map and are dropped;
          // the row and head coordinates are never negative (a TMA store must not start there)
          if (r == 0 && FFTS_IN_RANGE(t_half, p.L) && FFTS_IN_RANGE(hr, hcount)) {
            tma_store_3d(omap, stage_s, 64 * box, t_half, c.b * hcount + hr);
            bulk_commit();
          }
          if (role != 2) {
            // ---- pooling: thread r sums staged channel r % 64 of blocks r / 64, r / 64 + 2, ...
            const int ch = r & 63;
            const uint8_t *col = stage + (ch & 7) * 2;
            for (int pb = r >> 6; pb * p.bs < 128; pb += 2) {
              const int n = (t_half + pb * p.bs) / p.bs;
              if (n >= p.N) break;
              float s = 0.0f;
              const int r0 = pb * p.bs;
#pragma unroll 8
              for (int rr = r0; rr < r0 + p.bs; ++rr)
                s = __fadd_rn(s, __bfloat162float(
                                     *reinterpret_cast<const __nv_bfloat16 *>(col + rr * 128 + (((ch >> 3) ^ (rr & 7)) << 4))));
              if (FFTS_IN_RANGE(hr, hcount))
                p.pooled[role][((int64_t(c.b) * hcount + hr) * p.N + n) * kD + 64 * box + ch] =
                    __float2bfloat16_rn(__fdiv_rn(s, fbs));
            }
          }
          if (r == 0) bulk_wait_read();  // the store has read the box
          half_sync(half);               // before the next box overwrites it
        }
      }
    }
    if (r == 0) bulk_wait();  // this half's stores are complete before the CTA exits
    if (!ok) {
      *abort_flag = 1;
      atomicCAS(p.status, 0, kErrTimeoutEpilogue);
    }
  }

  // ---- teardown
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ----------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// bf16 rows of `inner` elements: dims {inner, rows, batch} (and a unit fourth dim
// when rank = 4), row / batch strides in elements, box {64, box_rows, 1(, 1)},
// SWIZZLE_128B; loads read out-of-range rows and columns as zero, stores drop them.
static int make_map(CUtensorMap *map, int rank, const void *base, int64_t inner, int64_t rows, int64_t batch,
                    int64_t ld, int64_t sb, int box_rows) {
  auto enc = get_encode();
  if (!enc) {
    set_error(FFTS_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
    return FFTS_E_CUDA;
  }
  cuuint64_t dims[4] = {cuuint64_t(inner), cuuint64_t(rows), cuuint64_t(batch), 1};
  cuuint64_t strides[3] = {cuuint64_t(ld) * 2, cuuint64_t(sb) * 2, cuuint64_t(sb) * 2 * cuuint64_t(batch)};
  cuuint32_t box[4] = {cuuint32_t(kBK), cuuint32_t(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult res = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cuuint32_t(rank), const_cast<void *>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) {
    set_error(FFTS_E_INVALID, "cuTensorMapEncodeTiled failed (%d): check 16-byte aligned base and strides", int(res));
    return FFTS_E_INVALID;
  }
  return FFTS_OK;
}

__device__ int g_qkv_status_sink;

}  // namespace qkv

int64_t qkv_workspace_bytes(int64_t L) {
  return L >= 1 ? ceil_div(L, 32) * 32 * qkv::kD * 2 * 2 : 0;  // cos and sin, rows padded to 32
}

int qkv_rope_pool(const void *x, int64_t B, int64_t L, int64_t K, int64_t x_ld, int64_t x_sb, const void *w,
                  int64_t w_ld, const void *bias, int64_t Hq, int64_t Hkv, int64_t D, const void *cos,
                  const void *sin, int64_t cs_ld, int bs, void *q_out, void *k_out, void *v_out, void *q_pooled,
                  void *k_pooled, void *raw, int64_t raw_ld, void *workspace, int64_t ws_bytes, int32_t *status,
                  cudaStream_t stream) {
  using namespace qkv;
  FFTS_REQUIRE(x && w && cos && sin && q_out && k_out && v_out && q_pooled && k_pooled,
               "qkv_rope_pool: NULL argument");
  FFTS_REQUIRE(D == kD, "qkv_rope_pool: head_dim must be %d (got %lld)", kD, (long long)D);
  FFTS_REQUIRE(bs == 16 || bs == 32 || bs == 64 || bs == 128, "qkv_rope_pool: block_size must be 16, 32, 64 or 128");
  FFTS_REQUIRE(B >= 1 && L >= 1 && K >= 1 && Hq >= 1 && Hkv >= 1, "qkv_rope_pool: empty or negative shape");
  const int64_t heads = Hq + 2 * Hkv;
  const int64_t m_tiles = ceil_div(L, kBM), n_tiles = ceil_div(heads * kD, kBN);
  FFTS_REQUIRE(L < (int64_t(1) << 31) && B * m_tiles * n_tiles < (int64_t(1) << 31) && heads < 65536,
               "qkv_rope_pool: shape too large");
  FFTS_REQUIRE(K % 8 == 0 && x_ld % 8 == 0 && x_ld >= K && w_ld % 8 == 0 && w_ld >= K && cs_ld % 8 == 0 &&
                   cs_ld >= D && (B == 1 || (x_sb % 8 == 0 && x_sb >= L * x_ld)),
               "qkv_rope_pool: K and the row strides must be multiples of 8 elements and cover their rows");
  FFTS_REQUIRE(!raw || (raw_ld % 8 == 0 && raw_ld >= heads * kD), "qkv_rope_pool: raw_ld too small or unaligned");
  if (workspace == nullptr || ws_bytes < qkv_workspace_bytes(L) || (reinterpret_cast<uintptr_t>(workspace) & 15)) {
    set_error(FFTS_E_WORKSPACE, "qkv_rope_pool: workspace needs %lld bytes, 16-byte aligned (got %lld)",
              (long long)qkv_workspace_bytes(L), (long long)ws_bytes);
    return FFTS_E_WORKSPACE;
  }
  for (const void *ptr : {x, w, bias, cos, sin, (const void *)q_out, (const void *)k_out, (const void *)v_out,
                          (const void *)q_pooled, (const void *)k_pooled, (const void *)raw})
    FFTS_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "qkv_rope_pool: pointers must be 16-byte aligned");
  CUtensorMap mx, mw, mq, mk, mv;
  int rc = make_map(&mx, 4, x, K, L, B, x_ld, B == 1 ? L * x_ld : x_sb, kBM);
  if (!rc) rc = make_map(&mw, 4, w, K, heads * kD, 1, w_ld, heads * kD * w_ld, kBN);
  // outputs [B * H, L, D]: a store box is 128 rows of one head, clipped at L
  if (!rc) rc = make_map(&mq, 3, q_out, kD, L, B * Hq, kD, L * kD, 128);
  if (!rc) rc = make_map(&mk, 3, k_out, kD, L, B * Hkv, kD, L * kD, 128);
  if (!rc) rc = make_map(&mv, 3, v_out, kD, L, B * Hkv, kD, L * kD, 128);
  if (rc) return rc;
  Params p{};
  p.bias = static_cast<const __nv_bfloat16 *>(bias);
  p.pooled[0] = static_cast<__nv_bfloat16 *>(q_pooled);
  p.pooled[1] = static_cast<__nv_bfloat16 *>(k_pooled);
  p.raw = static_cast<__nv_bfloat16 *>(raw);
  p.raw_ld = raw_ld;
  p.rope = static_cast<const uint4 *>(workspace);
  p.L = int(L);
  p.N = int(ceil_div(L, bs));
  p.Hq = int(Hq);
  p.Hkv = int(Hkv);
  p.heads = int(heads);
  p.bs = bs;
  p.kblocks = int(ceil_div(K, kBK));
  p.m_tiles = int(m_tiles);
  p.n_tiles = int(n_tiles);
  p.tiles = int(B * m_tiles * n_tiles);
  rc = device_wait_cycles(kWaitSeconds, &p.wait_cycles);
  if (!rc) rc = device_wait_cycles(kDrainSeconds, &p.drain_cycles);
  if (rc) return rc;
  if (status) {
    p.status = status;
  } else {
    void *sink = nullptr;
    FFTS_CUDA(cudaGetSymbolAddress(&sink, g_qkv_status_sink));
    p.status = static_cast<int *>(sink);
  }
  rc = ensure_func_smem(reinterpret_cast<const void *>(&qkv_rope_pool_kernel), Smem::bytes,
                        int(cudaSharedmemCarveoutMaxShared));
  if (rc) return rc;
  int sms = 0;
  rc = device_sm_count(&sms);
  if (rc) return rc;
  const int64_t rope_rows = ceil_div(L, 32) * 32;
  rope_tile_kernel<<<unsigned(ceil_div(rope_rows * 32, 256)), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(cos), static_cast<const __nv_bfloat16 *>(sin), cs_ld, L, rope_rows,
      static_cast<uint4 *>(workspace));
  FFTS_CUDA(cudaGetLastError());
  const unsigned grid = unsigned(p.tiles < sms ? p.tiles : sms);
  qkv_rope_pool_kernel<<<grid, kThreads, Smem::bytes, stream>>>(mx, mw, mq, mk, mv, p);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
