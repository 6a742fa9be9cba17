// ffts_common.cuh -- helpers shared by the FFTSparse sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <type_traits>

#include "../../include/fftsparse_b200.h"

namespace ffts {

// ------------------------------------------------------------ error state
void set_error(int code, const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);
// Raise func's dynamic shared-memory limit to at least bytes (and, if carveout >= 0,
// set its preferred carveout) on the current device; the attribute calls are made
// only when the value grows, so per-call launches skip them.
int ensure_func_smem(const void *func, int bytes, int carveout = -1);
// Properties of the current device, looked up once per device: its SM count and
// the number of SM clock cycles in `seconds` at its maximum SM clock (the bound
// of a kernel's spin-waits, which count cycles with clock64).
int device_sm_count(int *out);
int device_wait_cycles(double seconds, long long *out);

#define FFTS_REQUIRE(cond, ...)                          \
  do {                                                   \
    if (!(cond)) {                                       \
      ::ffts::set_error(FFTS_E_INVALID, __VA_ARGS__);    \
      return FFTS_E_INVALID;                             \
    }                                                    \
  } while (0)

#define FFTS_CUDA(call)                                           \
  do {                                                            \
    cudaError_t _e = (call);                                      \
    if (_e != cudaSuccess) return ::ffts::cuda_status(_e, #call); \
  } while (0)

// ------------------------------------------------------- element helpers
template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
  __device__ static inline float to_f32(float x) { return x; }
  __device__ static inline float from_f32(float x) { return x; }
  // value as stored in the dtype, returned as fp32 (identity for fp32)
  __device__ static inline float round_f32(float x) { return x; }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ static inline float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static inline __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
  __device__ static inline float round_f32(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

// Load 16 bytes and widen to fp32.
template <typename T>
__device__ inline void load_vec_f32(const T *p, float *out);

template <>
__device__ inline void load_vec_f32<float>(const float *p, float *out) {
  const float4 v = *reinterpret_cast<const float4 *>(p);
  out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}

template <>
__device__ inline void load_vec_f32<__nv_bfloat16>(const __nv_bfloat16 *p, float *out) {
  const uint4 v = *reinterpret_cast<const uint4 *>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Widen a 16-byte word of T to fp32.
template <typename T>
__device__ inline void widen_vec(const uint4 &v, float *out);

template <>
__device__ inline void widen_vec<float>(const uint4 &v, float *out) {
  out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
  out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}

template <>
__device__ inline void widen_vec<__nv_bfloat16>(const uint4 &v, float *out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Packed bf16 pairs in 32-bit registers: multiply and add with one
// round-to-nearest-even each (PTX mul.rn.bf16x2 / add.rn.bf16x2), and exact
// negation (sign bits flipped).
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_neg(uint32_t a) { return a ^ 0x80008000u; }

// Monotone 32-bit key of a float: larger value -> larger key; -0 maps to +0.
__device__ __forceinline__ uint32_t f32_key(float f) {
  if (f == 0.0f) f = 0.0f;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_f32(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

__host__ __device__ __forceinline__ int ilog2_ceil(int64_t m) {
  int r = 0;
  while ((int64_t(1) << r) < m) ++r;
  return r;
}

// ----------------------------------------------------- bounds-checked build
// Compute-sanitizer is not available where this library is tested, so the
// library has a second build, libfftsparse_b200_checked.so, compiled with
// -DFFTS_BOUNDS_CHECK.  In it, every FFTS_IN_RANGE(i, n) tests 0 <= i < n for an
// index whose value comes from data or from a ragged edge; a failed test counts
// itself in a word of this source file's own, remembers the line and the linear
// block index of the file's first failure, and evaluates to false so that the
// caller skips the access; FFTS_INDEX(i, n) records the same failure and yields
// index 0 instead, for a load the caller cannot skip.  Nothing traps.
// ffts_bounds_report() reads (and optionally clears) those words for the current
// device.  In the normal build the macro is the constant true and adds nothing.
#ifdef FFTS_BOUNDS_CHECK
namespace oob {
// per translation unit: first failure (bit 63 set | line << 32 | block index) and count
static __device__ unsigned long long g_first;
static __device__ unsigned int g_count;

static __device__ __noinline__ void note(int line) {
  const unsigned long long blk =
      blockIdx.x + (unsigned long long)gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z);
  atomicCAS(&g_first, 0ull, (1ull << 63) | ((unsigned long long)(line & 0x7fffffff) << 32) | (blk & 0xffffffffull));
  atomicAdd(&g_count, 1u);
}

static __device__ __forceinline__ bool in_range(long long i, long long n, int line) {
  const bool ok = i >= 0 && i < n;
  if (!ok) note(line);
  return ok;
}

// i when 0 <= i < n, else (after recording the failure) 0, a valid index of any
// non-empty extent: for loads whose address the caller cannot skip
static __device__ __forceinline__ long long checked_index(long long i, long long n, int line) {
  return in_range(i, n, line) ? i : 0;
}

// host side: this file's words, read (and zeroed if clear) on the current device
typedef int (*Reader)(int clear, unsigned long long *first, unsigned int *count);
void register_reader(const char *file, Reader fn);
static int read_words(int clear, unsigned long long *first, unsigned int *count) {
  cudaError_t e = cudaMemcpyFromSymbol(first, g_first, sizeof(*first));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(count, g_count, sizeof(*count));
  if (e == cudaSuccess && clear) {
    const unsigned long long z64 = 0;
    const unsigned int z32 = 0;
    e = cudaMemcpyToSymbol(g_first, &z64, sizeof(z64));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_count, &z32, sizeof(z32));
  }
  return e == cudaSuccess ? 0 : int(e);
}
static const bool g_registered = (register_reader(__BASE_FILE__, &read_words), true);
}  // namespace oob
#define FFTS_IN_RANGE(i, n) (::ffts::oob::in_range((long long)(i), (long long)(n), __LINE__))
#define FFTS_INDEX(i, n) \
  (static_cast<std::remove_cv_t<std::remove_reference_t<decltype(i)>>>( \
      ::ffts::oob::checked_index((long long)(i), (long long)(n), __LINE__)))
#else
#define FFTS_IN_RANGE(i, n) (true)
#define FFTS_INDEX(i, n) (i)
#endif

constexpr int kMaxBlocks = 4096;        // N limit (FFT size <= 8192)
constexpr int kMaxFFT = 8192;           // largest FFT length
constexpr int kDChunk = 8;              // channels per partial-spectrum CTA
constexpr int kLanes = 256;             // canonical reduction lanes

}  // namespace ffts
