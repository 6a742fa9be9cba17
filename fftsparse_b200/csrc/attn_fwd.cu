// attn_fwd.cu -- block-sparse causal attention forward on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the third-party block_sparse_attn_func (block_sparse_attn 0.0.2) as
// myattn_prefill calls it (attn_src/fft_attn/my_attn_v7.py:775-786): bf16
// q/k/v, fp32 accumulation, scale 1/sqrt(D), causal, head h uses mask plane h
// (head_mask_type all 1, :772), no dropout.  It reads q/k/v in their
// [B, H, L, D] layout through 4-D TMA descriptors (the reference copies them to
// [L, H, D] first, :528-530) and writes the output directly in the [B, L, H, D]
// layout the reference returns (:789-790).
//
// One CTA computes one 128-row query tile of one head, walking the selected
// key columns in 64-key tiles; two CTAs share an SM (256 TMEM columns and
// ~113 KB of shared memory each), so their pipelines interleave on the SM's
// tensor core:
//   warp 4      TMA producer: Q once, then the K tiles into a three-stage ring
//               and the V tiles into a two-stage ring (no multicast).
//   warp 5      MMA issuer (one thread): S = Q K^T into a double-buffered TMEM
//               accumulator (2 x 64 columns), O += P V with P read from TMEM;
//               completion is signalled with tcgen05.commit on mbarriers.
//   warps 0-3   softmax: thread r owns query row r (TMEM lane r); reads S(n)
//               while the tensor core computes S(n+1), applies the causal /
//               ragged / block masks, exponentiates against a running reference
//               max (rescaling O and l in TMEM only when a score outgrows it by
//               more than 2^64) and writes P as bf16 pairs over its S buffer;
//               finally normalises O, stages the bf16 tile in shared memory and
//               stores it row-contiguously to the output and to any peer GPUs'
//               buffers (the sharded prefill's all-gather).
// Unselected key tiles are never loaded.  Every mbarrier wait is bounded: on a
// time-out the CTA records an error status, stops issuing work, waits (bounded)
// for its own TMA copies and MMAs in flight, frees TMEM and exits.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "ffts_common.cuh"
#include "tc_sm100.cuh"

namespace ffts {
namespace attn {

constexpr int kBM = 128;       // query rows per CTA
constexpr int kBN = 64;        // key columns per tile
constexpr int kD = 128;        // head dim
constexpr int kThreads = 192;  // 6 warps; two CTAs share an SM
constexpr int kQBytes = kBM * kD * 2;        // 32 KB: two [128 rows][64 cols] swizzle boxes
constexpr int kQHalf = kQBytes / 2;
constexpr int kKVBytes = kBN * kD * 2;       // 16 KB: two [64 rows][64 cols] swizzle boxes
constexpr int kKVHalf = kKVBytes / 2;
constexpr int kMaxTiles = 4096;              // 64-key tiles per query tile (L <= 262144)
constexpr int kTileWords = kMaxTiles / 32;   // tile bitmask words
constexpr double kWaitSeconds = 2.0;   // bound on one wait (SM cycles at the device's clock, from the host)
constexpr double kDrainSeconds = 4.0;  // bound on draining own copies / MMAs

// status codes written to the caller's status word
constexpr int kErrTimeoutProducer = 1;
constexpr int kErrTimeoutMma = 2;
constexpr int kErrTimeoutSoftmax = 3;
constexpr int kErrSmemAlign = 4;  // dynamic shared memory not 1024-byte aligned: nothing was run

using namespace ::ffts::tc;  // PTX wrappers (tc_sm100.cuh)

// ------------------------------------------------------------------ layout
constexpr int kKStages = 3;     // K tile ring (a stage is released by the S MMA that read it)
constexpr int kVStages = 2;     // V tile ring (released by the PV MMA)
constexpr int kTmemCols = 256;  // S0, S1 (64 columns each) + O (128): two CTAs fill an SM's 512
constexpr uint32_t kTmemO = 128;
// P is kept <= 2^64 against the row's reference max: O and l are rescaled only
// when a row's scores outgrow it by that much (fp32 O stays far from overflow:
// < 2^64 * 2^18 keys * |v|)
constexpr float kRescaleLog2 = 64.0f;
constexpr float kPMax = 18446744073709551616.0f;  // 2^64

struct SmemLayout {
  // offsets from the dynamic shared memory base (1024-byte aligned, checked)
  static constexpr int q = 0;
  static constexpr int k = q + kQBytes;
  static constexpr int v = k + kKStages * kKVBytes;
  static constexpr int bars = v + kVStages * kKVBytes;
  static constexpr int nbars = 1 + 2 * kKStages + kVStages + 2 + 2 + 2 + 1;
  static constexpr int tmem_slot = bars + nbars * 8;
  static constexpr int misc = tmem_slot + 16;  // abort flag, tile count
  static constexpr int words = misc + 16;       // tile bitmask [kTileWords]
  static constexpr int end = words + kTileWords * 4;
  static constexpr int bytes = end;
};
// two CTAs per SM: 228 KB per SM, 1 KB of it reserved per CTA
static_assert(2 * (SmemLayout::bytes + 1024) <= 228 * 1024, "two CTAs must fit in an SM's shared memory");

// barrier indices
constexpr int BQ = 0;
constexpr int BKF = 1;                  // K full      [kKStages]
constexpr int BKE = BKF + kKStages;     // K empty     [kKStages]
constexpr int BVF = BKE + kKStages;     // V full      [kVStages]
constexpr int BSF = BVF + kVStages;     // S(n) in TMEM buffer n % 2 [2]
constexpr int BPV = BSF + 2;            // PV(n) complete, per S buffer n % 2 (also frees V stage n % 2) [2]
constexpr int BPF = BPV + 2;            // P(n) in TMEM, O rescaled, per S buffer n % 2 (128 arrivals) [2]
constexpr int BDRAIN = BPF + 2;
// Every ring of barriers above has one barrier per buffer because the softmax
// may run a full tile ahead of the MMA issuer (S(n+1) is computed before PV(n)
// is issued): with a single P barrier it could complete two phases before the
// issuer observes the first, and the parity wait would alias.

constexpr int kMaxPeerOut = 15;  // peer output buffers one launch also writes

struct Params {
  int B, H, Hkv, L, bs, bs_shift, causal;
  int nq;         // query tiles (128 rows) per head
  int nblk;       // mask blocks per row (N)
  int W;          // mask words per row
  const uint32_t *bits;
  __nv_bfloat16 *out;
  int64_t os_b, os_h, os_l;  // output strides (elements)
  int qt_lo, qt_cnt;         // query tiles [qt_lo, qt_lo + qt_cnt) are computed
  int out_row0;              // query row written at output row 0
  float scale_log2;
  int *status;
  long long wait_cycles;   // bound on one wait, SM cycles
  long long drain_cycles;  // bound on draining own copies / MMAs
  // Peer GPUs' output buffers (CUDA IPC mappings, same strides as out): every
  // output tile is also stored into each of them, so a sharded prefill's
  // all-gather rides on the epilogue over NVLink.
  int n_peers;
  __nv_bfloat16 *peer_out[kMaxPeerOut];
};

// Bits of 32 consecutive 64-key tiles [32*tw, 32*tw+32) of one mask row: a
// tile is kept if any mask block it overlaps is kept.
__device__ __forceinline__ uint32_t tile_word(const uint32_t *row, int W, int tw, int bs) {
  uint32_t out = 0;
  for (int t = 0; t < 32; ++t) {
    const int c0 = (tw * 32 + t) * kBN;            // first key of the tile
    const int b0 = c0 / bs, b1 = (c0 + kBN - 1) / bs;
    bool on = false;
    for (int blk = b0; blk <= b1; ++blk) {
      if ((blk >> 5) >= W) break;
      on |= (row[blk >> 5] >> (blk & 31)) & 1u;
    }
    out |= uint32_t(on) << t;
  }
  return out;
}

// Walks the set bits of the tile bitmask in increasing order; next() is called
// exactly once per selected tile, so it never reads past the last set bit.
struct TileCursor {
  const uint32_t *words;
  int w;
  uint32_t cur;
  __device__ explicit TileCursor(const uint32_t *wd) : words(wd), w(0), cur(wd[0]) {}
  __device__ __forceinline__ int next() {
    while (cur == 0) {
      if (!FFTS_IN_RANGE(w + 1, kTileWords)) return 0;  // more calls than set bits
      cur = words[++w];
    }
    const int t = __ffs(cur) - 1;
    cur &= cur - 1;
    return w * 32 + t;
  }
};

__global__ void __launch_bounds__(kThreads, 2)
    sparse_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Params prm) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  uint8_t *smem = smem_dyn;
  // SWIZZLE_128B TMA boxes and MMA descriptors need 1024-byte aligned tiles
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicCAS(prm.status, 0, kErrSmemAlign);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + SmemLayout::bars;
  auto bar = [&](int i) { return bar0 + 8u * uint32_t(i); };
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + SmemLayout::misc);
  int *ntiles_sh = reinterpret_cast<int *>(smem + SmemLayout::misc + 4);
  uint32_t *words = reinterpret_cast<uint32_t *>(smem + SmemLayout::words);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SmemLayout::tmem_slot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- tile coordinates: (b, kv head, query tile, head in group).  Query tiles
  // run heaviest (last) first, so the light ones fill the end of the grid.  When
  // the epilogue also pushes every tile to peers, the push volume per tile is
  // fixed while the causal work grows with the tile index: heavy and light tiles
  // then alternate (last, first, second last, second, ...), which spreads the
  // NVLink traffic over the whole kernel instead of bunching it where the light
  // tiles run.
  const int G = prm.H / prm.Hkv;
  int x = blockIdx.x;
  const int hg = x % G;
  x /= G;
  const int qi = x % prm.qt_cnt;
  const int qt = (prm.n_peers > 0 && (qi & 1)) ? prm.qt_lo + (qi >> 1)
                                               : prm.qt_lo + prm.qt_cnt - 1 - (prm.n_peers > 0 ? qi >> 1 : qi);
  x /= prm.qt_cnt;
  const int kvh = x % prm.Hkv;
  const int b = x / prm.Hkv;
  const int h = kvh * G + hg;
  const int rows_per_blk = prm.bs;                 // query rows per mask row
  const int mrows = (kBM + prm.bs - 1) / prm.bs;   // mask rows covered by this query tile

  // ---- setup: barriers, TMEM, tile list
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(bar(BQ), 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(bar(BKF + s), 1);
      mbar_init(bar(BKE + s), 1);
    }
    for (int s = 0; s < kVStages; ++s) mbar_init(bar(BVF + s), 1);
    mbar_init(bar(BSF), 1);
    mbar_init(bar(BSF + 1), 1);
    mbar_init(bar(BPV), 1);
    mbar_init(bar(BPV + 1), 1);
    mbar_init(bar(BPF), 128);
    mbar_init(bar(BPF + 1), 128);
    mbar_init(bar(BDRAIN), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == 4 && lane == 0) {
    prefetch_map(&tm_q);
    prefetch_map(&tm_k);
    prefetch_map(&tm_v);
  }
  // 64-key tiles to visit: OR over the mask rows of this query tile, causal cut.
  const int nkv_all = (prm.L + kBN - 1) / kBN;
  const int nkv = prm.causal ? min((qt + 1) * (kBM / kBN), nkv_all) : nkv_all;
  const int TW = (nkv + 31) / 32;
  if (warp == 0) {
    int base = 0;
    for (int c = 0; c < TW; c += 32) {
      const int tw = c + lane;
      uint32_t word = 0;
      if (tw < TW) {
        for (int s = 0; s < mrows; ++s) {
          const int mrow = qt * mrows + s;
          if (mrow < prm.nblk) {
            const uint32_t *row = prm.bits + ((int64_t(b) * prm.H + h) * prm.nblk + mrow) * prm.W;
            word |= tile_word(row, prm.W, tw, prm.bs);
          }
        }
        const int lim = nkv - tw * 32;  // tiles valid in this word
        if (lim < 32) word &= (lim <= 0) ? 0u : ((1u << lim) - 1u);
      }
      if (tw < TW && FFTS_IN_RANGE(tw, kTileWords)) words[tw] = word;
      int cnt = __popc(word);
      for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
      base += cnt;
    }
    if (lane == 0) *ntiles_sh = base;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = *ntiles_sh;
  const uint32_t tm_o = tmem + kTmemO;

  if (warp == 4) {
    // ================================================================ TMA producer
    // Q once; K(n+1) runs one tile ahead of V(n).  K(n) reuses the stage of
    // K(n-3), released by S(n-3); V(n) the stage of V(n-2), released by PV(n-2).
    if (lane == 0 && ntiles > 0) {
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      mbar_arrive_tx(bar(BQ), kQBytes);
      tma_load_4d(sbase + SmemLayout::q, &tm_q, bar(BQ), 0, qt * kBM, h, b);
      tma_load_4d(sbase + SmemLayout::q + kQHalf, &tm_q, bar(BQ), 64, qt * kBM, h, b);
      TileCursor kcur(words), vcur(words);
      auto load = [&](int n, bool is_k) -> bool {
        const int ns = is_k ? kKStages : kVStages;
        const int s = n % ns;
        // a K stage is free once S(n-3) has completed (its empty barrier), a V
        // stage once PV(n-2) has (the PV barrier of that buffer): the phase the
        // V wait names is the latest one, since PV(n) needs the copy issued here
        const int full = (is_k ? BKF : BVF) + s, empty = (is_k ? BKE : BPV) + s;
        if (!mbar_wait(bar(empty), ((n / ns) & 1) ^ 1, abort_flag, prm.wait_cycles)) return false;
        mbar_arrive_tx(bar(full), kKVBytes);
        const uint32_t dst = sbase + (is_k ? SmemLayout::k : SmemLayout::v) + s * kKVBytes;
        const CUtensorMap *map = is_k ? &tm_k : &tm_v;
        const int j = FFTS_INDEX(is_k ? kcur.next() : vcur.next(), nkv);
        tma_load_4d(dst, map, bar(full), 0, j * kBN, kvh, b);
        tma_load_4d(dst + kKVHalf, map, bar(full), 64, j * kBN, kvh, b);
        if (is_k) ++issued_k; else ++issued_v;
        return true;
      };
      ok = load(0, true);
      for (int n = 0; n < ntiles && ok; ++n) {
        if (n + 1 < ntiles) ok = load(n + 1, true);
        if (ok) ok = load(n, false);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicCAS(prm.status, 0, kErrTimeoutProducer);
        // wait (bounded, ignoring the abort flag) for the copies this thread issued
        volatile int never = 0;
        mbar_wait(bar(BQ), 0, &never, prm.drain_cycles);
        for (int n = max(0, issued_k - kKStages); n < issued_k; ++n)
          mbar_wait(bar(BKF + n % kKStages), (n / kKStages) & 1, &never, prm.drain_cycles);
        for (int n = max(0, issued_v - 2); n < issued_v; ++n)
          mbar_wait(bar(BVF + n % 2), (n >> 1) & 1, &never, prm.drain_cycles);
      }
    }
  } else if (warp == 5) {
    // ================================================================ MMA issuer
    // S(0), S(1), then per tile n: PV(n) (after P(n)), S(n+2).  S(n+2) overwrites
    // the TMEM buffer that held P(n); tcgen05.mma operations of one thread
    // execute in issue order, so PV(n) has read P(n) by then.
    if (lane == 0 && ntiles > 0) {
      const uint32_t idS = idesc_bf16(false, kBN), idPV = idesc_bf16(true, kD);
      bool ok = mbar_wait(bar(BQ), 0, abort_flag, prm.wait_cycles);
      fence_after();
      // Shared-memory descriptors of the tile bases; a 16-byte multiple offset
      // within shared memory adds (offset >> 4) to the address field, which
      // cannot carry out of its 14 bits below 256 KB.
      const uint64_t dq = smem_desc(sbase + SmemLayout::q, 16, 1024);
      const uint64_t dk0 = smem_desc(sbase + SmemLayout::k, 16, 1024);
      const uint64_t dv0 = smem_desc(sbase + SmemLayout::v, kKVHalf, 1024);
      auto issue_s = [&](int n) -> bool {
        const int s = n % 2, ks = n % kKStages;
        if (!mbar_wait(bar(BKF + ks), (n / kKStages) & 1, abort_flag, prm.wait_cycles)) return false;
        fence_after();
        const uint64_t dk = dk0 + uint64_t((ks * kKVBytes) >> 4);
        const uint32_t td = tmem + s * kBN;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t qoff = (kk >> 2) * kQHalf + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * kKVHalf + (kk & 3) * 32;
          umma_f16(td, dq + (qoff >> 4), dk + (koff >> 4), idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar(BSF + s));
        umma_commit(bar(BKE + ks));
        return true;
      };
      auto issue_pv = [&](int m) -> bool {
        const int s = m % 2;
        if (!mbar_wait(bar(BVF + s), (m >> 1) & 1, abort_flag, prm.wait_cycles)) return false;
        if (!mbar_wait(bar(BPF + s), (m >> 1) & 1, abort_flag, prm.wait_cycles)) return false;
        fence_after();
        const uint64_t dv = dv0 + uint64_t((s * kKVBytes) >> 4);
        const uint32_t pt = tmem + s * kBN;  // P(m): bf16 pairs in the first 32 columns of S buffer m % 2
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          umma_f16_ts(tm_o, pt + kk * 8, dv + uint64_t((kk * 2048) >> 4), idPV, (m > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar(BPV + s));
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && ntiles > 1) ok = issue_s(1);
      for (int n = 0; n < ntiles && ok; ++n) {
        ok = issue_pv(n);
        if (ok && n + 2 < ntiles) ok = issue_s(n + 2);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicCAS(prm.status, 0, kErrTimeoutMma);
      }
      // drain: wait (bounded) until every MMA this thread issued has completed
      umma_commit(bar(BDRAIN));
      volatile int never = 0;
      mbar_wait(bar(BDRAIN), 0, &never, prm.drain_cycles);
    }
  } else {
    // ================================================================ softmax (warps 0-3)
    const int r = threadIdx.x;  // query row within the tile == TMEM lane
    const int row_g = qt * kBM + r;
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    // m_ref: the max the current P and O are scaled to (lags the true max by < 2^64 in P)
    float m_ref = -INFINITY, l_run = 0.0f;
    bool ok = true;
    const int mrow = min(qt * mrows + r / rows_per_blk, prm.nblk - 1);
    const uint32_t *rowbits = prm.bits + ((int64_t(b) * prm.H + h) * prm.nblk + mrow) * prm.W;
    const float2 sc2 = make_float2(prm.scale_log2, prm.scale_log2);
    TileCursor cur(words);
    for (int n = 0; n < ntiles; ++n) {
      const int sb = n % 2;
      const int j = FFTS_INDEX(cur.next(), nkv);
      if (!__all_sync(0xffffffffu, mbar_wait(bar(BSF + sb), (n >> 1) & 1, abort_flag, prm.wait_cycles))) { ok = false; break; }
      fence_after();
      const uint32_t s_addr = tmem + sb * kBN + lane_off;
      // masks: causal diagonal, ragged end, and (block_size < 128) this row's own
      // mask row; whole 32-column words since block_size >= 32
      const int col0 = j * kBN;
      const bool edge = (prm.causal && col0 + kBN - 1 > qt * kBM) || col0 + kBN > prm.L || prm.bs < kBM;
      uint32_t kw[2] = {0xffffffffu, 0xffffffffu};
      if (edge) {
        int lim = min(kBN, prm.L - col0);
        if (prm.causal) lim = min(lim, row_g - col0 + 1);
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const int rem = lim - 32 * w;
          uint32_t m = rem >= 32 ? 0xffffffffu : (rem <= 0 ? 0u : ((1u << rem) - 1u));
          if (prm.bs < kBM) {
            const int blk = (col0 + 32 * w) >> prm.bs_shift;
            if (blk >= prm.nblk || !((rowbits[FFTS_INDEX(blk >> 5, prm.W)] >> (blk & 31)) & 1u)) m = 0u;
          }
          kw[w] = m;
        }
      }
      float x[kBN];
      tmem_ld32(s_addr, x);
      tmem_wait_ld();
      tmem_ld32(s_addr + 32, x + 32);  // lands while the first half is processed
      if (edge) {
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (!((kw[0] >> c) & 1u)) x[c] = -INFINITY;
      }
      // P = exp2(s*scale - m_ref) as bf16 pairs over the first 32 columns of this
      // S buffer (the columns already read).  The common path takes m_ref as it
      // stands, without this tile's max, and keeps the result when every P of
      // the row is <= 2^kRescaleLog2 (checked on the tile's row sum).  A row's
      // first valid tile, or a tile whose P would exceed that, takes the max
      // path: new m_ref, O and l rescaled by alpha, P recomputed.
      float2 rs2[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
      float alpha = 1.0f;
      bool fast = !__any_sync(0xffffffffu, m_ref == -INFINITY);
      auto exp_half = [&](int cc, float2 off2) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int c = cc * 32 + e;
          const float2 a = __ffma2_rn(make_float2(x[c], x[c + 1]), sc2, off2);
          float2 ex;
          ex.x = fast_exp2(a.x);
          ex.y = fast_exp2(a.y);
          rs2[(e >> 1) & 1] = __fadd2_rn(rs2[(e >> 1) & 1], ex);
          const __nv_bfloat162 pr = __floats2bfloat162_rn(ex.x, ex.y);
          pk[e >> 1] = *reinterpret_cast<const uint32_t *>(&pr);
        }
        tmem_st16u(s_addr + cc * 16, pk);
      };
      if (fast) {
        const float moff = m_ref * prm.scale_log2;
        exp_half(0, make_float2(-moff, -moff));
        tmem_wait_ld();
        if (edge) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (!((kw[1] >> c) & 1u)) x[32 + c] = -INFINITY;
        }
        exp_half(1, make_float2(-moff, -moff));
        const float tsum = (rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y);
        if (__any_sync(0xffffffffu, !(tsum <= kPMax))) {
          fast = false;
          tmem_wait_st();  // the max path below rewrites P
          rs2[0] = rs2[1] = make_float2(0.0f, 0.0f);
        }
      } else {
        tmem_wait_ld();
        if (edge) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (!((kw[1] >> c) & 1u)) x[32 + c] = -INFINITY;
        }
      }
      if (!fast) {
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < kBN; c += 2) mx4[(c >> 1) & 3] = max3f(mx4[(c >> 1) & 3], x[c], x[c + 1]);
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        const bool grow = mx > m_ref && (m_ref == -INFINITY || (mx - m_ref) * prm.scale_log2 > kRescaleLog2);
        if (grow) {
          alpha = m_ref == -INFINITY ? 0.0f : fast_exp2((m_ref - mx) * prm.scale_log2);
          m_ref = mx;
        }
        const float moff = (m_ref == -INFINITY ? 0.0f : m_ref) * prm.scale_log2;
        exp_half(0, make_float2(-moff, -moff));
        exp_half(1, make_float2(-moff, -moff));
      }
      const float2 rsum = __fadd2_rn(rs2[0], rs2[1]);
      l_run = l_run * alpha + (rsum.x + rsum.y);
      tmem_wait_st();
      if (n >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // O must hold PV(n-1) before it is rescaled.  PV(n-1) completes the
        // barrier of S buffer (n-1) % 2; that barrier's previous phase (PV(n-3))
        // is complete and its next (PV(n+1)) needs P(n+1), so the parity is exact.
        if (!__all_sync(0xffffffffu,
                        mbar_wait(bar(BPV + (n - 1) % 2), ((n - 1) >> 1) & 1, abort_flag, prm.wait_cycles))) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(tm_o + lane_off + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 v = __fmul2_rn(make_float2(o[e], o[e + 1]), make_float2(alpha, alpha));
            o[e] = v.x;
            o[e + 1] = v.y;
          }
          tmem_st32(tm_o + lane_off + c * 32, o);
        }
        tmem_wait_st();
      }
      fence_before();
      mbar_arrive(bar(BPF + sb));
    }
    // O is final once PV(ntiles-1) has completed (its commit also covers every
    // earlier MMA).  Its buffer's barrier has completed PV(ntiles-3) and has no
    // later phase, so the parity is exact.
    if (ok && ntiles > 0) {
      const int m = ntiles - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar(BPV + m % 2), (m >> 1) & 1, abort_flag, prm.wait_cycles));
    }
    if (!ok) {
      *abort_flag = 1;
      atomicCAS(prm.status, 0, kErrTimeoutSoftmax);
    }
    fence_after();
    // epilogue: O / l -> bf16 -> out[b, row, h, :] (and the same rows of every
    // peer buffer).  The bf16 tile is staged in the Q tile's shared memory: with
    // ok, every MMA has completed (the last PV commit covers them all) and no
    // copy is in flight, and with no tiles Q was never loaded.  Row r's 16-byte
    // chunk j sits at r * 256 + ((j ^ (r & 15)) << 4), so the row-per-thread
    // writes and the row-contiguous reads below are both free of bank conflicts.
    const int tile_rows = min(kBM, prm.L - qt * kBM);
    const float inv_l = (ok && l_run > 0.0f) ? 1.0f / l_run : 0.0f;
    uint8_t *stage = smem + SmemLayout::q;
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        if (ntiles > 0) {
          tmem_ld32(tm_o + lane_off + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0.0f;
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 pr =
                __floats2bfloat162_rn(o[q4 * 8 + 2 * e] * inv_l, o[q4 * 8 + 2 * e + 1] * inv_l);
            w[e] = *reinterpret_cast<const uint32_t *>(&pr);
          }
          const int j = c * 4 + q4;
          *reinterpret_cast<uint4 *>(stage + r * 256 + ((j ^ (r & 15)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    // every softmax thread arrives here; the tile is copied out only if all four
    // warps completed (ok is uniform within a warp, not across the warps)
    int all_ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(all_ok)
        : "r"(int(ok))
        : "memory");
    if (all_ok) {
      // each warp instruction stores two whole 256-byte rows
      const int64_t off = int64_t(b) * prm.os_b + int64_t(qt * kBM - prm.out_row0) * prm.os_l + int64_t(h) * prm.os_h;
      // the peers in an order rotated per CTA, so that the CTAs' stores spread
      // over all peers rather than reaching them one at a time
      const int rot = prm.n_peers > 0 ? int(blockIdx.x % unsigned(prm.n_peers)) : 0;
#pragma unroll 1
      for (int d = -1; d < prm.n_peers; ++d) {
        int pd = d + rot;
        if (pd >= prm.n_peers) pd -= prm.n_peers;
        __nv_bfloat16 *base = (d < 0 ? prm.out : prm.peer_out[pd]) + off;
#pragma unroll 4
        for (int k = r; k < tile_rows * 16; k += kBM) {
          const int row = k >> 4, j = k & 15;
          const uint4 val = *reinterpret_cast<const uint4 *>(stage + row * 256 + ((j ^ (row & 15)) << 4));
          if (FFTS_IN_RANGE(qt * kBM + row, prm.L) && FFTS_IN_RANGE(qt * kBM + row - prm.out_row0, prm.L))
            *reinterpret_cast<uint4 *>(base + int64_t(row) * prm.os_l + j * 8) = val;
        }
      }
      // the peers learn of these rows from a flag a later kernel on this
      // stream stores; make them visible system-wide before the CTA retires
      if (prm.n_peers > 0) __threadfence_system();
    } else if (row_g < prm.L) {
      // after a time-out copies may still land in shared memory: zeros, row per thread
      __nv_bfloat16 *dst =
          prm.out + int64_t(b) * prm.os_b + int64_t(row_g - prm.out_row0) * prm.os_l + int64_t(h) * prm.os_h;
#pragma unroll
      for (int c = 0; c < 16; ++c) *reinterpret_cast<uint4 *>(dst + c * 8) = make_uint4(0u, 0u, 0u, 0u);
    }
  }

  // ---- teardown
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 5) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ----------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

static int make_map(CUtensorMap *map, const void *base, int64_t L, int64_t Hx, int64_t B, const int64_t *st,
                    int box_rows) {
  auto enc = get_encode();
  if (!enc) {
    set_error(FFTS_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
    return FFTS_E_CUDA;
  }
  cuuint64_t dims[4] = {cuuint64_t(kD), cuuint64_t(L), cuuint64_t(Hx), cuuint64_t(B)};
  cuuint64_t strides[3] = {cuuint64_t(st[2]) * 2, cuuint64_t(st[1]) * 2, cuuint64_t(st[0]) * 2};
  cuuint32_t box[4] = {64, cuuint32_t(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(FFTS_E_INVALID, "cuTensorMapEncodeTiled failed (%d): check 16-byte aligned base and strides", int(r));
    return FFTS_E_INVALID;
  }
  return FFTS_OK;
}

__device__ int g_attn_status_sink;

}  // namespace attn

int sparse_attn_fwd(const void *q, const void *k, const void *v, int64_t B, int64_t H, int64_t Hkv, int64_t L,
                    int64_t D, const int64_t *qs, const int64_t *ks, const int64_t *vs, const uint32_t *bits, int bs,
                    int causal, void *out, const int64_t *os, int64_t row_lo, int64_t row_hi,
                    void *const *peer_out, int n_peers, int32_t *status, cudaStream_t stream) {
  using namespace attn;
  FFTS_REQUIRE(q && k && v && bits && out && qs && ks && vs && os, "sparse_attn: NULL argument");
  FFTS_REQUIRE(D == kD, "sparse_attn: head_dim must be 128 (got %lld)", (long long)D);
  FFTS_REQUIRE(bs == 32 || bs == 64 || bs == 128, "sparse_attn: block_size must be 32, 64 or 128 (got %d)", bs);
  FFTS_REQUIRE(B >= 1 && H >= 1 && Hkv >= 1 && H % Hkv == 0 && L >= 1, "sparse_attn: bad shape");
  const int64_t nblk = ceil_div(L, bs);
  const int64_t nq = ceil_div(L, kBM);
  FFTS_REQUIRE(nblk <= kMaxBlocks && ceil_div(L, kBN) <= kMaxTiles, "sparse_attn: sequence too long for the tile list");
  FFTS_REQUIRE(L < (int64_t(1) << 31) && B * H * nq < (int64_t(1) << 31), "sparse_attn: grid too large");
  for (const int64_t *st : {qs, ks, vs})
    FFTS_REQUIRE(st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0 && st[2] >= D,
                 "sparse_attn: q/k/v strides must be multiples of 8 elements (16 bytes)");
  FFTS_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(k) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(v) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0,
               "sparse_attn: tensors must be 16-byte aligned");
  FFTS_REQUIRE(os[0] % 8 == 0 && os[1] % 8 == 0 && os[2] % 8 == 0, "sparse_attn: output strides must be 16-byte multiples");
  FFTS_REQUIRE(row_lo >= 0 && row_lo < row_hi && row_hi <= L && row_lo % kBM == 0 && (row_hi % kBM == 0 || row_hi == L),
               "sparse_attn: query rows [%lld, %lld) must lie in [0, L) on %d-row boundaries", (long long)row_lo,
               (long long)row_hi, kBM);
  FFTS_REQUIRE(n_peers >= 0 && n_peers <= kMaxPeerOut && (n_peers == 0 || peer_out),
               "sparse_attn: at most %d peer outputs", kMaxPeerOut);
  for (int i = 0; i < n_peers; ++i)
    FFTS_REQUIRE(peer_out[i] && (reinterpret_cast<uintptr_t>(peer_out[i]) & 15) == 0,
                 "sparse_attn: peer output %d must be non-NULL and 16-byte aligned", i);
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, q, L, H, B, qs, kBM);
  if (!rc) rc = make_map(&mk, k, L, Hkv, B, ks, kBN);
  if (!rc) rc = make_map(&mv, v, L, Hkv, B, vs, kBN);
  if (rc) return rc;
  Params p{};
  p.B = int(B); p.H = int(H); p.Hkv = int(Hkv); p.L = int(L); p.bs = bs; p.causal = causal ? 1 : 0;
  p.bs_shift = bs == 32 ? 5 : (bs == 64 ? 6 : 7);
  p.nq = int(nq); p.nblk = int(nblk); p.W = int(ceil_div(nblk, 32));
  p.bits = bits;
  p.out = static_cast<__nv_bfloat16 *>(out);
  p.os_b = os[0]; p.os_h = os[1]; p.os_l = os[2];
  p.qt_lo = int(row_lo / kBM);
  p.qt_cnt = int(ceil_div(row_hi, kBM) - row_lo / kBM);
  p.out_row0 = int(row_lo);
  p.scale_log2 = float(1.4426950408889634 / sqrt(double(D)));
  rc = device_wait_cycles(kWaitSeconds, &p.wait_cycles);
  if (!rc) rc = device_wait_cycles(kDrainSeconds, &p.drain_cycles);
  if (rc) return rc;
  p.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i) p.peer_out[i] = static_cast<__nv_bfloat16 *>(peer_out[i]);
  if (status) {
    p.status = status;
  } else {
    void *sink = nullptr;
    FFTS_CUDA(cudaGetSymbolAddress(&sink, g_attn_status_sink));
    p.status = static_cast<int *>(sink);
  }
  // the largest shared-memory carveout, so that two CTAs fit on an SM
  rc = ensure_func_smem(reinterpret_cast<const void *>(&sparse_attn_kernel), SmemLayout::bytes,
                        int(cudaSharedmemCarveoutMaxShared));
  if (rc) return rc;
  const unsigned grid = unsigned(B * H * p.qt_cnt);
  sparse_attn_kernel<<<grid, kThreads, SmemLayout::bytes, stream>>>(mq, mk, mv, p);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
