// peer.cu -- the sharded prefill's output all-gather on the GPUs' copy engines.
//
// With the path sharded by KV group, every rank computes the attention output of
// its heads and every rank needs all heads (o_proj consumes them).  NCCL's
// all-gather runs as SM kernels and cannot start while the attention kernel holds
// every SM (its CTAs use all shared memory and TMEM), so a gather issued beside
// the next row chunk's attention does not overlap it.  These entry points let
// the host side (fftsparse_b200/dist.py, PeerGather) push each finished row chunk
// straight into the peers' output buffers with cudaMemcpy2DAsync over NVLink: the
// copy engines move the data while the SMs compute the next chunk.  Each peer's
// copies go on a stream of their own, so that the pushes to different peers run
// side by side on different copy engines (one stream's copies run one at a time).
//
//   ffts_ipc_handle / ffts_ipc_open / ffts_ipc_close  map a peer's buffer (CUDA
//       IPC; the offset of the buffer inside its allocation travels with the
//       handle, so buffers from torch's caching allocator work);
//   ffts_copy_rows   one strided copy (height rows of width bytes, same pitch on
//       both sides) to each of n destinations, copy i on stream i, each stream
//       first waiting for an event (the chunk's attention) when one is given;
//   ffts_copy_2d     one pitched copy in any direction (host <-> device), for
//       the host-buffer prefill's per-chunk read-back of its head columns;
//   ffts_signal      a small kernel storing an epoch number into flags with
//       release semantics at system scope, flag i queued on stream i after the
//       copies there (one launch per run of flags that share a stream);
//   ffts_wait_flags  a one-warp kernel that waits, with acquire loads, until every
//       flag holds at least the epoch; the wait is bounded (about 2 s of SM
//       cycles) and on a time-out writes status 5 and returns.
//
// Peers' memory is only ever touched by copy engines and by the flag stores: no
// TMA copy, and no multicast, reads another GPU's memory.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "ffts_common.cuh"

namespace ffts {
namespace peer {

constexpr double kWaitSeconds = 2.0;  // bound on the flag wait (converted to SM cycles per device)
constexpr int kErrPeerTimeout = 5;

constexpr int kMaxPeers = 32;

struct FlagList {
  int32_t *flag[kMaxPeers];
};

__global__ void signal_kernel(FlagList flags, int n, int32_t value) {
  if (int(threadIdx.x) < n)
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.flag[threadIdx.x]), "r"(value) : "memory");
}

__global__ void wait_kernel(const int32_t *flags, int n, int32_t epoch, int32_t *status, long long limit) {
  const int i = threadIdx.x;
  if (i >= n) return;
  const long long t0 = clock64();
  while (true) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
    if (v >= epoch) break;
    if (clock64() - t0 > limit) {
      atomicCAS(status, 0, kErrPeerTimeout);
      break;
    }
    __nanosleep(256);
  }
}

static PFN_cuMemGetAddressRange_v3020 get_range() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }
  return fn;
}

}  // namespace peer
}  // namespace ffts

using namespace ffts;

extern "C" {

FFTS_API int32_t ffts_ipc_handle(const void *ptr, void *handle, int64_t *offset) {
  FFTS_REQUIRE(ptr && handle && offset, "ipc_handle: NULL argument");
  auto range = peer::get_range();
  if (!range) {
    set_error(FFTS_E_CUDA, "cuMemGetAddressRange is unavailable");
    return FFTS_E_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error(FFTS_E_INVALID, "ipc_handle: %p is not device memory", ptr);
    return FFTS_E_INVALID;
  }
  cudaIpcMemHandle_t h;
  FFTS_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)));
  memcpy(handle, &h, sizeof(h));
  *offset = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return FFTS_OK;
}

FFTS_API int32_t ffts_ipc_open(const void *handle, int64_t offset, void **ptr) {
  FFTS_REQUIRE(handle && ptr && offset >= 0, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  FFTS_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<char *>(base) + offset;
  return FFTS_OK;
}

FFTS_API int32_t ffts_ipc_close(void *ptr, int64_t offset) {
  FFTS_REQUIRE(ptr && offset >= 0, "ipc_close: bad argument");
  FFTS_CUDA(cudaIpcCloseMemHandle(static_cast<char *>(ptr) - offset));
  return FFTS_OK;
}

FFTS_API int32_t ffts_copy_2d(void *dst, int64_t dst_pitch, const void *src, int64_t src_pitch, int64_t width,
                              int64_t height, void *stream) {
  FFTS_REQUIRE(dst && src && width > 0 && height > 0 && dst_pitch >= width && src_pitch >= width,
               "copy_2d: bad argument");
  FFTS_CUDA(cudaMemcpy2DAsync(dst, size_t(dst_pitch), src, size_t(src_pitch), size_t(width), size_t(height),
                              cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return FFTS_OK;
}

FFTS_API int32_t ffts_copy_rows(void *const *dsts, void *const *streams, int32_t n, const void *src, int64_t pitch,
                                int64_t width, int64_t height, void *after) {
  FFTS_REQUIRE(dsts && streams && src && n >= 0 && width > 0 && height > 0 && pitch >= width,
               "copy_rows: bad argument");
  for (int i = 0; i < n; ++i) {
    FFTS_REQUIRE(dsts[i], "copy_rows: NULL destination %d", i);
    const cudaStream_t st = static_cast<cudaStream_t>(streams[i]);
    if (after) FFTS_CUDA(cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(after), 0));
    FFTS_CUDA(cudaMemcpy2DAsync(dsts[i], size_t(pitch), src, size_t(pitch), size_t(width), size_t(height),
                                cudaMemcpyDeviceToDevice, st));
  }
  return FFTS_OK;
}

FFTS_API int32_t ffts_signal(int32_t *const *flags, void *const *streams, int32_t n, int32_t value) {
  FFTS_REQUIRE(flags && streams && n >= 1 && n <= 1024, "signal: bad argument");
  for (int i = 0; i < n;) {
    peer::FlagList fl{};
    int c = 0;
    for (; i + c < n && c < peer::kMaxPeers && streams[i + c] == streams[i]; ++c) {
      int32_t *f = flags[i + c];
      FFTS_REQUIRE(f && (reinterpret_cast<uintptr_t>(f) & 3) == 0, "signal: bad flag address");
      fl.flag[c] = f;
    }
    peer::signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(streams[i])>>>(fl, c, value);
    FFTS_CUDA(cudaGetLastError());
    i += c;
  }
  return FFTS_OK;
}

FFTS_API int32_t ffts_wait_flags(const int32_t *flags, int32_t n, int32_t epoch, int32_t *status, void *stream) {
  FFTS_REQUIRE(flags && status && n >= 1 && n <= 32, "wait_flags: bad argument");
  long long limit = 0;
  const int rc = device_wait_cycles(peer::kWaitSeconds, &limit);
  if (rc) return rc;
  peer::wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, n, epoch, status, limit);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // extern "C"
