// Allocation-free C entry point: bias gradient (column sum of a bf16 matrix).
//
// This entry point has no counterpart in the reference library, which has no
// native code at all; it exists for C callers of this library.
//
// Who it is for: code that calls into this library but may not allocate
// device memory itself.  Typical cases are a plugin or custom op hosted by
// another runtime that owns every device allocation and gives its plugins a
// fixed budget, a service that has reserved the whole device for its own
// memory pool, and latency-critical loops that cannot afford cudaMalloc /
// cudaFree (both can block until the device is idle).  Such a caller still
// owns and passes the input and the output; the kernel's scratch (the fp32
// per-block partial sums) comes from a fixed array compiled into this
// library instead of from an allocator.
//
// Contract:
//   * scratch is a file-scope `static __device__` array of kMaxScratchFloats
//     floats (8 MiB).  Every GPU that loads this library holds it until the
//     process exits.  A call needs ceil(rows / 128) * cols floats of it;
//     larger problems are rejected with status 2 and a message, never
//     clipped.
//   * the array's name is only a host-side stand-in: host code must not
//     hand it to a kernel.  The device address is obtained with
//     cudaGetSymbolAddress once per CUDA context (each device's primary
//     context, or a context the host runtime created), with that context
//     current, on the first call made in it.  That first call therefore does
//     the set-up (and may initialise the device's primary context); make it
//     before any latency-sensitive section.
//   * problems with more than 65,535 bands of 128 rows are handled by CTAs
//     that walk several bands; the scratch need and the limit are the same.
//   * every call shares the one array, and each call overwrites every
//     partial it reads before reading it, so nothing has to start at zero.
//     Calls whose kernels can overlap on the GPU (different streams, or
//     different host threads) race on the array: serialise them, e.g. by
//     issuing them on one stream.
//   * no cudaMalloc, cudaFree or allocating library routine is called.
//
// The exported C interface (prototypes, return codes, the scratch limit) is
// declared in csrc/include/mnb_noalloc.h, which this file includes so the
// definitions below are checked against it.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../include/mnb_noalloc.h"

namespace {

constexpr long long kMaxScratchFloats = MNB_NOALLOC_MAX_SCRATCH_FLOATS;  // 8 MiB
constexpr int kRowsPerBlock = 128;
// gridDim.y limit: problems with more 128-row bands than this run each CTA
// row over several bands (one partial per band, as with fewer bands).
constexpr long long kMaxGridY = 65535;
constexpr int kMaxContexts = 64;

static __device__ __align__(256) float g_colsum_scratch[kMaxScratchFloats];

// The array has its own device address in every CUDA context (the primary
// context of each device, and any context a host runtime creates with
// cuCtxCreate), so the looked-up address is cached per context.
struct ScratchAddr {
  CUcontext ctx;
  float* addr;
};
ScratchAddr g_scratch_addr[kMaxContexts] = {};
int g_scratch_count = 0;
std::mutex g_setup_mutex;
thread_local char g_last_error[256] = "";

int fail(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, float* f) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&ws[j]);
    const float2 t = __bfloat1622float2(b);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

// Partial column sums: band b covers rows [128b, 128b+128); block (x, y)
// handles 256 columns of bands y, y + gridDim.y, ... and writes one partial
// row per band, so the scratch layout does not depend on the grid.
__global__ void __launch_bounds__(256) noalloc_colsum_partials(const __nv_bfloat16* __restrict__ g,
                                                               float* __restrict__ scratch, int rows, int cols,
                                                               int bands) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int c0 = blockIdx.x * 256 + lane * 8;
  for (int band = blockIdx.y; band < bands; band += gridDim.y) {
    const int r0 = band * kRowsPerBlock;
    const int r1 = min(rows, r0 + kRowsPerBlock);
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (c0 < cols) {
      for (int r = r0 + warp; r < r1; r += 8) {
        float f[8];
        load8_bf16(g + static_cast<long long>(r) * cols + c0, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] += f[j];
      }
    }
    __syncthreads();  // the previous band's reads of `red` are done
#pragma unroll
    for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = s[j];
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
    const int c = blockIdx.x * 256 + threadIdx.x;
    if (c < cols) scratch[static_cast<long long>(band) * cols + c] = t;
  }
}

__global__ void noalloc_fold(const float* __restrict__ scratch, int parts, int cols, void* out, int out_f32,
                             int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += scratch[static_cast<long long>(p) * cols + c];
  if (out_f32) {
    float* o = static_cast<float*>(out);
    o[c] = accumulate ? o[c] + s : s;
  } else {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
    o[c] = __float2bfloat16_rn(accumulate ? __bfloat162float(o[c]) + s : s);
  }
}

// Device address of the scratch array in the current CUDA context, looked up
// once per context with that context current.
// cuCtxGetCurrent, resolved through the runtime (the library does not link
// libcuda directly, so it still loads on a machine without a driver).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

int scratch_for_current_context(float** out) {
  const CtxGetCurrentFn get_ctx = ctx_get_current();
  if (get_ctx == nullptr) return fail(3, "cuCtxGetCurrent is not available from the CUDA driver");
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return fail(3, "cuCtxGetCurrent failed");
  if (ctx == nullptr) {
    // No context yet on this thread: make the current device's primary
    // context current (cudaSetDevice initialises it), as the runtime would.
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 == cudaSuccess) e0 = cudaSetDevice(dev);
    if (e0 != cudaSuccess) return fail(3, cudaGetErrorString(e0));
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return fail(3, "no current CUDA context");
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  for (int i = 0; i < g_scratch_count; ++i) {
    if (g_scratch_addr[i].ctx == ctx) {
      *out = g_scratch_addr[i].addr;
      return 0;
    }
  }
  if (g_scratch_count == kMaxContexts) return fail(3, "too many CUDA contexts for the scratch address cache");
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_colsum_scratch);
  if (e != cudaSuccess || p == nullptr) return fail(3, cudaGetErrorString(e));
  g_scratch_addr[g_scratch_count++] = {ctx, static_cast<float*>(p)};
  *out = static_cast<float*>(p);
  return 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) const char* mnb_noalloc_last_error() { return g_last_error; }

extern "C" __attribute__((visibility("default"))) long long mnb_noalloc_max_scratch_floats() {
  return kMaxScratchFloats;
}

extern "C" __attribute__((visibility("default"))) int mnb_bias_grad_noalloc(const void* grad, void* out, int rows,
                                                                            int cols, int out_is_fp32,
                                                                            int accumulate, void* stream) {
  if (grad == nullptr || out == nullptr) return fail(1, "grad and out must be device pointers");
  if (rows < 1 || cols < 1 || cols % 8 != 0) return fail(1, "rows >= 1 and cols a positive multiple of 8 required");
  if (reinterpret_cast<uintptr_t>(grad) % 16 != 0) return fail(1, "grad must be 16-byte aligned");
  const long long parts = (static_cast<long long>(rows) + kRowsPerBlock - 1) / kRowsPerBlock;
  const long long need = parts * static_cast<long long>(cols);
  if (need > kMaxScratchFloats) {
    char msg[160];
    std::snprintf(msg, sizeof(msg), "problem needs %lld scratch floats; the built-in maximum is %lld", need,
                  kMaxScratchFloats);
    return fail(2, msg);
  }
  float* scratch = nullptr;
  const int rc = scratch_for_current_context(&scratch);
  if (rc != 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid_y = static_cast<unsigned>(parts < kMaxGridY ? parts : kMaxGridY);
  noalloc_colsum_partials<<<dim3((cols + 255) / 256, grid_y), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(grad), scratch, rows, cols, static_cast<int>(parts));
  noalloc_fold<<<(cols + 255) / 256, 256, 0, s>>>(scratch, static_cast<int>(parts), cols, out, out_is_fp32 ? 1 : 0,
                                                  accumulate ? 1 : 0);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(3, cudaGetErrorString(e));
  g_last_error[0] = '\0';
  return 0;
}
