// noalloc.cu -- block-mask selection that needs no device allocation at all.
//
// ffts_block_mask asks its caller for a device workspace (about 4 MB at 128K
// tokens and 32 heads).  Some callers cannot provide one: an inference engine
// that reserves all of a GPU's memory for its own pool at start-up and forbids
// later cudaMalloc calls, or a framework plugin whose per-request hook is not
// allowed to allocate because cudaMalloc may synchronise the whole device and
// stall every other stream.  ffts_block_mask_noalloc serves those callers: it
// runs the same kernels as ffts_block_mask on a scratch array that is part of
// the library's own device image.
//
// The scratch is one file-scope __device__ array of kScratchBytes (8 MiB).  Each
// GPU that loads the library keeps it resident until the process exits.  Host
// code cannot use the array's name as a device address (it names a host-side
// shadow), so the first call on each device looks up the real address with
// cudaGetSymbolAddress while that device is current, and every later call on
// that device reuses it.  Because that first call does this set-up (and may
// upload the library's constant tables), make the first call on a device before
// any stream capture.
//
// Every call on a device shares the same scratch and leaves its contents
// behind.  Nothing in it has to start at zero: each call writes every scratch
// word it later reads.  Two calls whose kernels overlap on the GPU (for example
// on two streams of the same device) race on the scratch and corrupt each
// other's results; serialise them.

#include <mutex>

#include "ffts_common.cuh"

namespace ffts {

int64_t mask_workspace_bytes(int64_t B, int64_t H, int64_t N, int64_t D);
int block_mask(const void *qb, const void *kb, int dtype, int64_t B, int64_t H, int64_t Hkv, int64_t D,
               const ffts_mask_params *params, uint32_t *bits, int32_t *row_count, float *corr, float *csum,
               uint8_t *is_stripe, float *svar, void *workspace, int64_t ws_bytes, cudaStream_t stream);

namespace {

constexpr int64_t kScratchBytes = int64_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_mask_scratch[kScratchBytes];

std::mutex g_scratch_mutex;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of g_mask_scratch on the current device (looked up once per device).
int scratch_address(void **out) {
  int dev = 0;
  FFTS_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error(FFTS_E_DEVICE, "device ordinal %d beyond the %d devices this entry point tracks", dev, kMaxDevices);
    return FFTS_E_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_mask_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_mask_scratch)");
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return FFTS_OK;
}

}  // namespace
}  // namespace ffts

extern "C" FFTS_API int32_t ffts_block_mask_noalloc(const void *qb, const void *kb, int32_t dtype, int64_t B,
                                                     int64_t H, int64_t Hkv, int64_t D,
                                                     const ffts_mask_params *params, uint32_t *mask_bits,
                                                     int32_t *row_count, float *corr, float *corr_sum,
                                                     uint8_t *is_stripe, float *stripe_var, void *stream) {
  using namespace ffts;
  FFTS_REQUIRE(params != nullptr, "ffts_block_mask_noalloc: params is NULL");
  FFTS_REQUIRE(B >= 1 && H >= 1 && D >= 1 && params->n_blocks >= 1, "ffts_block_mask_noalloc: empty shape");
  int dev = 0, major = 0;
  FFTS_CUDA(cudaGetDevice(&dev));
  FFTS_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  if (major != 10) {
    set_error(FFTS_E_DEVICE, "device %d has compute capability %d.x; this library targets sm_100a", dev, major);
    return FFTS_E_DEVICE;
  }
  const int64_t need = mask_workspace_bytes(B, H, params->n_blocks, D);
  if (need > kScratchBytes) {
    set_error(FFTS_E_WORKSPACE,
              "ffts_block_mask_noalloc: B=%lld H=%lld N=%d D=%lld needs %lld bytes of scratch, more than the "
              "library's fixed %lld-byte scratch; use ffts_block_mask with a caller workspace",
              (long long)B, (long long)H, params->n_blocks, (long long)D, (long long)need,
              (long long)kScratchBytes);
    return FFTS_E_WORKSPACE;
  }
  void *scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  return block_mask(qb, kb, dtype, B, H, Hkv, D, params, mask_bits, row_count, corr, corr_sum, is_stripe,
                    stripe_var, scratch, kScratchBytes, static_cast<cudaStream_t>(stream));
}
