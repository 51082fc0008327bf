// Memory-bound kernels of the GPT training step, all bf16 in/out with fp32 math:
// LayerNorm forward/backward, GELU, token+position embedding forward/backward,
// softmax cross-entropy (loss and logit gradient in one pass), column sums for
// bias gradients, and a multi-tensor AdamW with fp32 master weights.
//
// Row kernels use one warp per row with 16-byte vector accesses; reductions
// over rows (LayerNorm weight grads, bias grads) write per-block fp32 partials
// that a second small kernel folds, so results do not depend on atomics.
#include <map>
#include <mutex>
#include <tuple>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace mnb {

namespace {

constexpr int kRowWarps = 8;  // rows per block in the warp-per-row kernels

MNB_DEVICE void load8(const __nv_bfloat16* p, float* f) {
  uint4 w = ld_v4(p);
  uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = unpack_bf16x2(ws[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}
MNB_DEVICE void store8(__nv_bfloat16* p, const float* f) {
  st_v4(p, make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7])));
}

}  // namespace

// ---------------------------------------------------------------------------
// LayerNorm
// ---------------------------------------------------------------------------
__global__ void layernorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                     const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                     float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int C,
                                     float eps) {
  const int row = blockIdx.x * kRowWarps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + static_cast<long long>(row) * C;
  float s = 0.f;
  for (int c = lane * 8; c < C; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += f[j];
  }
  const float mean = warp_sum(s) / C;
  float ss = 0.f;
  for (int c = lane * 8; c < C; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float d = f[j] - mean;
      ss += d * d;
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / C + eps);
  __nv_bfloat16* yr = y + static_cast<long long>(row) * C;
  for (int c = lane * 8; c < C; c += 256) {
    float f[8], g[8], h[8];
    load8(xr + c, f);
    load8(w + c, g);
    load8(b + c, h);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = (f[j] - mean) * rstd * g[j] + h[j];
    store8(yr + c, f);
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// LayerNorm forward with the row in registers (C = NCH * 256): one read of x,
// mean and variance from registers (two-pass, exact), w and b loaded once per
// warp for all the rows it visits (grid-stride).
template <int NCH>
__global__ void __launch_bounds__(256, 2) layernorm_fwd_reg_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const __nv_bfloat16* __restrict__ w,
                                                                const __nv_bfloat16* __restrict__ b,
                                                                __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out,
                                                                float* __restrict__ rstd_out, int rows, float eps) {
  constexpr int C = NCH * 256;
  const int lane = threadIdx.x % 32;
  const int warps = gridDim.x * (blockDim.x / 32);
  float ww[NCH][8], bb[NCH][8];
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    load8(w + k * 256 + lane * 8, ww[k]);
    load8(b + k * 256 + lane * 8, bb[k]);
  }
  for (int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; row < rows; row += warps) {
    const __nv_bfloat16* xr = x + static_cast<long long>(row) * C;
    float f[NCH][8];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      load8(xr + k * 256 + lane * 8, f[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += f[k][j];
    }
    const float mean = warp_sum(s) * (1.f / C);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = f[k][j] - mean;
        ss += d * d;
      }
    const float rstd = rsqrtf(warp_sum(ss) * (1.f / C) + eps);
    __nv_bfloat16* yr = y + static_cast<long long>(row) * C;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (f[k][j] - mean) * rstd * ww[k][j] + bb[k][j];
      store8(yr + k * 256 + lane * 8, o);
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

// Wide rows (C = 8 * blockDim.x, up to 4096): one block per row, 8 columns per thread.
__global__ void __launch_bounds__(512) layernorm_fwd_wide_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 const __nv_bfloat16* __restrict__ w,
                                                                 const __nv_bfloat16* __restrict__ b,
                                                                 __nv_bfloat16* __restrict__ y,
                                                                 float* __restrict__ mean_out,
                                                                 float* __restrict__ rstd_out, int rows, int C,
                                                                 float eps) {
  __shared__ float red[2][16];
  const int c0 = threadIdx.x * 8;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  float ww[8], bb[8];
  load8(w + c0, ww);
  load8(b + c0, bb);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long off = static_cast<long long>(row) * C + c0;
    float f[8];
    load8(x + off, f);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += f[j];
    s = warp_sum(s);
    if (lane == 0) red[0][warp] = s;
    __syncthreads();
    float mean = 0.f;
    for (int i = 0; i < nw; ++i) mean += red[0][i];
    mean /= C;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = f[j] - mean;
      ss += d * d;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[1][warp] = ss;
    __syncthreads();
    float var = 0.f;
    for (int i = 0; i < nw; ++i) var += red[1][i];
    const float rstd = rsqrtf(var / C + eps);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = (f[j] - mean) * rstd * ww[j] + bb[j];
    store8(y + off, o);
    if (threadIdx.x == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
    __syncthreads();  // red[] is rewritten by the next row
  }
}

// Grid-wide column sums without a second kernel.  `acc` is a persistent fp32
// accumulator of n values followed by one u32 arrival counter, all zero
// between calls: every block adds its partial sums atomically, and the last
// block to arrive writes the results (bf16 or fp32, optionally accumulating)
// and zeroes the accumulator and the counter again.  Calls that share `acc`
// must be ordered (one stream).
MNB_DEVICE void finish_fold(float* acc, int n, void* out0, void* out1, int split, int out_f32, int accumulate) {
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* counter = reinterpret_cast<unsigned int*>(acc + n);
    last = atomicAdd(counter, 1u) == gridDim.x * gridDim.y - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = *reinterpret_cast<volatile float*>(acc + i);
    acc[i] = 0.f;
    void* out = i < split ? out0 : out1;
    const int k = i < split ? i : i - split;
    if (out_f32) {
      float* o = reinterpret_cast<float*>(out) + k;
      *o = accumulate ? *o + v : v;
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + k;
      *o = f32_to_bf16(accumulate ? bf16_to_f32(*o) + v : v);
    }
  }
  if (threadIdx.x == 0) *reinterpret_cast<unsigned int*>(acc + n) = 0u;
}
// Shared-memory partials of one block -> the accumulator, then finish.
MNB_DEVICE void fold_into(float* acc, const float* sacc, int n, void* out0, void* out1, int split, int out_f32,
                          int accumulate) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) atomicAdd(acc + i, sacc[i]);
  finish_fold(acc, n, out0, out1, split, out_f32, accumulate);
}

// dx per row; per-block fp32 partials of dgamma/dbeta in `part` [gridDim.x, 2, C].
// NCH > 0: the row (C = NCH*256 wide) stays in registers, one global read,
// and each lane accumulates the weight gradients of its own columns in
// registers across all rows it visits.  NCH == 0: any C, shared-memory atomics.
template <int NCH>
__global__ void __launch_bounds__(256, 1) layernorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                     const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean,
                                     const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                     float* __restrict__ part, int rows, int C, void* out_dw, void* out_db,
                                     int out_f32, int accumulate) {
  extern __shared__ float sacc[];  // [2][C]
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) sacc[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x % 32;
  const int warp = threadIdx.x / 32;
  if constexpr (NCH > 0) {
    float dg[NCH][8], dbb[NCH][8], ww[NCH][8];
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      load8(w + k * 256 + lane * 8, ww[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) dg[k][j] = dbb[k][j] = 0.f;
    }
    // PR rows per pass (2 while registers allow): their loads are all in
    // flight before the first reduction
    constexpr int PR = NCH <= 3 ? 2 : 1;
    const int stride = gridDim.x * kRowWarps;
    for (int row0 = blockIdx.x * kRowWarps + warp; row0 < rows; row0 += PR * stride) {
      float xh[PR][NCH][8], g[PR][NCH][8];
      float mu[PR], rs[PR];
#pragma unroll
      for (int p = 0; p < PR; ++p) {
        const int row = row0 + p * stride;
        if (row < rows) {
          const __nv_bfloat16* xr = x + static_cast<long long>(row) * C;
          const __nv_bfloat16* gr = dy + static_cast<long long>(row) * C;
          mu[p] = mean[row];
          rs[p] = rstd[row];
#pragma unroll
          for (int k = 0; k < NCH; ++k) {
            load8(xr + k * 256 + lane * 8, xh[p][k]);
            load8(gr + k * 256 + lane * 8, g[p][k]);
          }
        }
      }
#pragma unroll
      for (int p = 0; p < PR; ++p) {
        const int row = row0 + p * stride;
        if (row >= rows) break;
        float a = 0.f, bsum = 0.f;
#pragma unroll
        for (int k = 0; k < NCH; ++k)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            xh[p][k][j] = (xh[p][k][j] - mu[p]) * rs[p];
            const float d = g[p][k][j] * ww[k][j];
            a += d;
            bsum += d * xh[p][k][j];
            dg[k][j] += g[p][k][j] * xh[p][k][j];
            dbb[k][j] += g[p][k][j];
          }
        a = warp_sum(a) / C;
        bsum = warp_sum(bsum) / C;
        __nv_bfloat16* dr = dx + static_cast<long long>(row) * C;
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
          float o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = rs[p] * (g[p][k][j] * ww[k][j] - a - xh[p][k][j] * bsum);
          store8(dr + k * 256 + lane * 8, o);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < NCH; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        atomicAdd(&sacc[k * 256 + lane * 8 + j], dg[k][j]);
        atomicAdd(&sacc[C + k * 256 + lane * 8 + j], dbb[k][j]);
      }
  } else {
    for (int row = blockIdx.x * kRowWarps + warp; row < rows; row += gridDim.x * kRowWarps) {
      const __nv_bfloat16* xr = x + static_cast<long long>(row) * C;
      const __nv_bfloat16* gr = dy + static_cast<long long>(row) * C;
      const float mu = mean[row], rs = rstd[row];
      float a = 0.f, bsum = 0.f;
      for (int c = lane * 8; c < C; c += 256) {
        float f[8], g[8], wv[8];
        load8(xr + c, f);
        load8(gr + c, g);
        load8(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float xhv = (f[j] - mu) * rs;
          float d = g[j] * wv[j];
          a += d;
          bsum += d * xhv;
          atomicAdd(&sacc[c + j], g[j] * xhv);
          atomicAdd(&sacc[C + c + j], g[j]);
        }
      }
      a = warp_sum(a) / C;
      bsum = warp_sum(bsum) / C;
      __nv_bfloat16* dr = dx + static_cast<long long>(row) * C;
      for (int c = lane * 8; c < C; c += 256) {
        float f[8], g[8], wv[8], o[8];
        load8(xr + c, f);
        load8(gr + c, g);
        load8(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float xhv = (f[j] - mu) * rs;
          o[j] = rs * (g[j] * wv[j] - a - xhv * bsum);
        }
        store8(dr + c, o);
      }
    }
  }
  __syncthreads();
  fold_into(part, sacc, 2 * C, out_dw, out_db, C, out_f32, accumulate);
}

// Same result as layernorm_bwd_kernel<NCH> (C = NCH * 256), with the x and dy
// rows brought into shared memory by bulk (TMA) copies DEPTH rows ahead of
// each warp: a warp keeps DEPTH rows (DEPTH x 2 x C x 2 bytes) in flight
// instead of the two it can hold in registers, which is what reaching HBM
// bandwidth takes at one CTA per SM.  Each warp owns a private ring of DEPTH
// row slots with one mbarrier per slot; lane 0 refills a slot once the warp
// has consumed it.  dgamma / dbeta as in the register kernel.
MNB_DEVICE void ld_shared_bf16x8(uint32_t addr, float* f) {
  uint32_t w0, w1, w2, w3;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3) : "r"(addr));
  const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = unpack_bf16x2(ws[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

// ADD: dx also receives `add` (the gradient reaching x through a residual
// branch), so autograd needs no separate accumulation kernel; a slot then
// holds three rows (x, dy, add).
template <int NCH, int DEPTH, bool ADD = false>
constexpr size_t ln_bwd_bulk_smem() {
  return static_cast<size_t>(kRowWarps) * DEPTH * (ADD ? 3 : 2) * 2 * NCH * 256 + 2 * NCH * 256 * 4 +
         kRowWarps * DEPTH * 8 + 128;
}

template <int NCH, int DEPTH, bool ADD = false>
__global__ void __launch_bounds__(256, 1)
    layernorm_bwd_bulk_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                              const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean,
                              const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                              float* __restrict__ part, int rows, int Cdyn, void* out_dw, void* out_db, int out_f32,
                              int accumulate, const __nv_bfloat16* __restrict__ add = nullptr) {
  constexpr int C = NCH * 256;
  constexpr uint32_t kRowBytes = C * 2;
  constexpr int kSlotRows = ADD ? 3 : 2;
  extern __shared__ uint8_t ln_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ln_raw) + 127) & ~uintptr_t(127));
  float* sacc = reinterpret_cast<float*>(base + kRowWarps * DEPTH * kSlotRows * kRowBytes);  // [2][C]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sacc + 2 * C);                       // [warps][DEPTH]
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) sacc[i] = 0.f;
  if (threadIdx.x < kRowWarps * DEPTH) mbar_init(smem_u32(bars + threadIdx.x), 1);
  fence_mbar_init();
  __syncthreads();
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const uint32_t wbuf = smem_u32(base) + warp * DEPTH * kSlotRows * kRowBytes;
  const uint32_t wbar = smem_u32(bars + warp * DEPTH);
  const int stride = gridDim.x * kRowWarps;
  const int first = blockIdx.x * kRowWarps + warp;
  const int n_mine = first < rows ? (rows - first + stride - 1) / stride : 0;
  auto issue = [&](int k) {  // lane 0: rows of this warp's k-th turn into slot k % DEPTH
    const long long row = first + static_cast<long long>(k) * stride;
    const uint32_t dst = wbuf + (k % DEPTH) * kSlotRows * kRowBytes, bar = wbar + 8 * (k % DEPTH);
    mbar_arrive_expect_tx(bar, kSlotRows * kRowBytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(x + row * C), "r"(kRowBytes), "r"(bar) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst + kRowBytes), "l"(dy + row * C), "r"(kRowBytes), "r"(bar) : "memory");
    if constexpr (ADD)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"(dst + 2 * kRowBytes), "l"(add + row * C), "r"(kRowBytes), "r"(bar) : "memory");
  };
  if (lane == 0)
    for (int k = 0; k < DEPTH && k < n_mine; ++k) issue(k);
  float dg[NCH][8], dbb[NCH][8], ww[NCH][8];
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    load8(w + k * 256 + lane * 8, ww[k]);
#pragma unroll
    for (int j = 0; j < 8; ++j) dg[k][j] = dbb[k][j] = 0.f;
  }
  // lane i holds the statistics of this warp's turn 32 * m + i: one load
  // latency per 32 rows instead of one per row
  float mu_l = 0.f, rs_l = 0.f;
#pragma unroll 1
  for (int k = 0; k < n_mine; ++k) {
    const int row = first + k * stride;
    if (k % 32 == 0 && k + lane < n_mine) {
      const int r = first + (k + lane) * stride;
      mu_l = mean[r];
      rs_l = rstd[r];
    }
    const float mu = __shfl_sync(0xffffffffu, mu_l, k % 32), rs = __shfl_sync(0xffffffffu, rs_l, k % 32);
    if (!__all_sync(0xffffffffu, mbar_wait(wbar + 8 * (k % DEPTH), (k / DEPTH) & 1, nullptr))) break;
    const uint32_t src = wbuf + (k % DEPTH) * kSlotRows * kRowBytes;
    float xh[NCH][8], g[NCH][8], ad[ADD ? NCH : 1][8];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      ld_shared_bf16x8(src + (c * 256 + lane * 8) * 2, xh[c]);
      ld_shared_bf16x8(src + kRowBytes + (c * 256 + lane * 8) * 2, g[c]);
      if constexpr (ADD) ld_shared_bf16x8(src + 2 * kRowBytes + (c * 256 + lane * 8) * 2, ad[c]);
    }
    float a = 0.f, bsum = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xh[c][j] = (xh[c][j] - mu) * rs;
        const float d = g[c][j] * ww[c][j];
        a += d;
        bsum += d * xh[c][j];
        dg[c][j] += g[c][j] * xh[c][j];
        dbb[c][j] += g[c][j];
      }
    // every lane's reads of this slot are complete (their values were used
    // above; the add row's values are consumed by the adds below, which the
    // fence and refill can only follow once those loads have returned)
    if constexpr (ADD) {
#pragma unroll
      for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int j = 0; j < 8; ++j) asm volatile("" ::"f"(ad[c][j]));
    }
    __syncwarp();
    if (lane == 0 && k + DEPTH < n_mine) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(k + DEPTH);
    }
    a = warp_sum(a) / C;
    bsum = warp_sum(bsum) / C;
    __nv_bfloat16* dr = dx + static_cast<long long>(row) * C;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rs * (g[c][j] * ww[c][j] - a - xh[c][j] * bsum);
      if constexpr (ADD) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += ad[c][j];
      }
      store8(dr + c * 256 + lane * 8, o);
    }
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      atomicAdd(&sacc[c * 256 + lane * 8 + j], dg[c][j]);
      atomicAdd(&sacc[C + c * 256 + lane * 8 + j], dbb[c][j]);
    }
  __syncthreads();
  fold_into(part, sacc, 2 * C, out_dw, out_db, C, out_f32, accumulate);
}

// Wide rows (C = 8 * blockDim.x, e.g. 2048 / 4096): one block per row, each
// thread owns 8 columns; the two row sums go through a block reduction, and
// each thread keeps its columns' weight-gradient sums in registers across
// the rows its block visits.  Per-block partials as above.
__global__ void __launch_bounds__(512) layernorm_bwd_wide_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ mean, const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ part, int rows, int C, void* out_dw, void* out_db, int out_f32, int accumulate) {
  __shared__ float red[2][16][2];
  const int c0 = threadIdx.x * 8;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  float ww[8], dg[8], dbb[8];
  load8(w + c0, ww);
#pragma unroll
  for (int j = 0; j < 8; ++j) dg[j] = dbb[j] = 0.f;
  int par = 0;
  for (int row = blockIdx.x; row < rows; row += gridDim.x, par ^= 1) {
    const long long off = static_cast<long long>(row) * C + c0;
    float xh[8], g[8];
    load8(x + off, xh);
    load8(dy + off, g);
    const float mu = mean[row], rs = rstd[row];
    float a = 0.f, bsum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      xh[j] = (xh[j] - mu) * rs;
      const float d = g[j] * ww[j];
      a += d;
      bsum += d * xh[j];
      dg[j] += g[j] * xh[j];
      dbb[j] += g[j];
    }
    a = warp_sum(a);
    bsum = warp_sum(bsum);
    if (lane == 0) {
      red[par][warp][0] = a;
      red[par][warp][1] = bsum;
    }
    __syncthreads();  // double-buffered by row parity: one barrier per row
    a = 0.f;
    bsum = 0.f;
    for (int i = 0; i < nw; ++i) {
      a += red[par][i][0];
      bsum += red[par][i][1];
    }
    a /= C;
    bsum /= C;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = rs * (g[j] * ww[j] - a - xh[j] * bsum);
    store8(dx + off, o);
  }
  // this block's column sums into the shared accumulator; the last block finishes
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    atomicAdd(part + c0 + j, dg[j]);
    atomicAdd(part + C + c0 + j, dbb[j]);
  }
  finish_fold(part, 2 * C, out_dw, out_db, C, out_f32, accumulate);
}

// out[c] (+)= sum over `nparts` rows of part[:, c]; bf16 or fp32 destination.
// Block = 32 columns x 8 warps; warp w sums parts w, w+8, ... and the 8 warp
// sums are combined in shared memory, so long part lists stay parallel.
__global__ void __launch_bounds__(256) fold_partials_kernel(const float* __restrict__ part, int nparts,
                                                            long long stride, int C, void* out, int out_f32,
                                                            int accumulate) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int c = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < C) {
#pragma unroll 4
    for (int p = warp; p < nparts; p += 8) s += part[p * stride + c];
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp != 0 || c >= C) return;
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w][lane];
  if (out_f32) {
    float* o = reinterpret_cast<float*>(out);
    o[c] = accumulate ? o[c] + t : t;
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
    o[c] = f32_to_bf16(accumulate ? bf16_to_f32(o[c]) + t : t);
  }
}

// Column sums of a [rows, C] bf16 matrix into per-block partials [gridDim.y, C].
// A block covers 256 columns x kColRows rows: each warp walks every 8th row
// with 16-byte loads into register accumulators, then the 8 warps are summed
// through shared memory.
constexpr int kColRows = 128;
__global__ void __launch_bounds__(256) colsum_partial_kernel(const __nv_bfloat16* __restrict__ g,
                                                             float* __restrict__ part, int rows, int C) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * kColRows;
  const int r1 = min(rows, r0 + kColRows);
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c0 < C) {
#pragma unroll 4
    for (int r = r0 + warp; r < r1; r += 8) {
      float f[8];
      load8(g + static_cast<long long>(r) * C + c0, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] += f[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = s[j];
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < C) part[static_cast<long long>(blockIdx.y) * C + c] = t;
}

// ---------------------------------------------------------------------------
// GELU (standalone; the MLP path fuses it into the GEMM epilogues)
// ---------------------------------------------------------------------------
__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n8) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float f[8];
    load8(x + 8 * i, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = gelu_exact(f[j]);
    store8(y + 8 * i, f);
  }
}
__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                                __nv_bfloat16* __restrict__ dx, long long n8) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float f[8], g[8];
    load8(x + 8 * i, f);
    load8(dy + 8 * i, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = g[j] * gelu_grad(f[j]);
    store8(dx + 8 * i, f);
  }
}

// ---------------------------------------------------------------------------
// Embedding: y[b, t] = wte[idx[b, t]] + wpe[t]
// ---------------------------------------------------------------------------
__global__ void embed_fwd_kernel(const int64_t* __restrict__ idx, const __nv_bfloat16* __restrict__ wte,
                                 const __nv_bfloat16* __restrict__ wpe, __nv_bfloat16* __restrict__ y, int tokens,
                                 int T, int C) {
  const int row = blockIdx.x * kRowWarps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= tokens) return;
  const long long tok = idx[row];
  const int t = row % T;
  for (int c = lane * 8; c < C; c += 256) {
    float a[8], p[8];
    load8(wte + tok * C + c, a);
    load8(wpe + static_cast<long long>(t) * C + c, p);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] += p[j];
    store8(y + static_cast<long long>(row) * C + c, a);
  }
}

// dwte[idx] += dy (bf16x2 atomics, collisions are rare for real token streams);
__global__ void embed_bwd_tok_kernel(const int64_t* __restrict__ idx, const __nv_bfloat16* __restrict__ dy,
                                     __nv_bfloat16* __restrict__ dwte, int tokens, int C) {
  const int row = blockIdx.x * kRowWarps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= tokens) return;
  const long long tok = idx[row];
  for (int c = lane * 2; c < C; c += 64) {
    __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(dy + static_cast<long long>(row) * C + c);
    atomicAdd(reinterpret_cast<__nv_bfloat162*>(dwte + tok * C + c), g);
  }
}

// dwpe[t] (+)= sum_b dy[b, t]
__global__ void embed_bwd_pos_kernel(const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dwpe, int B,
                                     int T, int C, int accumulate) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < C; c += blockDim.x * 8) {
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < B; ++b) {
      float f[8];
      load8(dy + (static_cast<long long>(b) * T + t) * C + c, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] += f[j];
    }
    if (accumulate) {
      float o[8];
      load8(dwpe + static_cast<long long>(t) * C + c, o);
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] += o[j];
    }
    store8(dwpe + static_cast<long long>(t) * C + c, s);
  }
}

// ---------------------------------------------------------------------------
// Cross-entropy: per row, loss = logsumexp(z) - z[target]; the logits are
// overwritten in place with (softmax(z) - onehot) * grad_scale.
// ---------------------------------------------------------------------------
constexpr int kXentThreads = 512;

__global__ void __launch_bounds__(kXentThreads) xent_fwd_bwd_kernel(__nv_bfloat16* __restrict__ logits,
                                                                    const int64_t* __restrict__ targets,
                                                                    float* __restrict__ loss, int V, long long ld,
                                                                    float grad_scale, int ignore_index) {
  __shared__ float sm[32], ss[32];
  const int row = blockIdx.x;
  __nv_bfloat16* z = logits + static_cast<long long>(row) * ld;
  // Online max / sum of exp per thread, then merged across the block.
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += kXentThreads * 8) {
    float f[8];
    if (c + 8 <= V) {
      load8(z + c, f);
    } else {
      for (int j = 0; j < 8; ++j) f[j] = (c + j < V) ? bf16_to_f32(z[c + j]) : -INFINITY;
    }
    float lm = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, f[j]);
    float nm = fmaxf(m, lm);
    float acc = (m == -INFINITY) ? 0.f : s * __expf(m - nm);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += (f[j] == -INFINITY) ? 0.f : __expf(f[j] - nm);
    m = nm;
    s = acc;
  }
  // warp merge
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float om = __shfl_xor_sync(0xffffffffu, m, o);
    float os = __shfl_xor_sync(0xffffffffu, s, o);
    float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < kXentThreads / 32 ? sm[lane] : -INFINITY;
    s = lane < kXentThreads / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float om = __shfl_xor_sync(0xffffffffu, m, o);
      float os = __shfl_xor_sync(0xffffffffu, s, o);
      float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (lane == 0) {
      sm[0] = m;
      ss[0] = s;
    }
  }
  __syncthreads();
  const float rmax = sm[0];
  const float inv = 1.f / ss[0];
  const int64_t tgt = targets[row];
  const bool ignored = tgt == ignore_index;
  if (threadIdx.x == 0) {
    loss[row] = ignored ? 0.f : (rmax + logf(ss[0]) - bf16_to_f32(z[tgt]));
  }
  __syncthreads();  // everyone read z[tgt] above before it is overwritten
  const float gs = ignored ? 0.f : grad_scale;
  for (int c = threadIdx.x * 8; c < V; c += kXentThreads * 8) {
    if (c + 8 <= V) {
      float f[8];
      load8(z + c, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float p = __expf(f[j] - rmax) * inv;
        f[j] = (p - ((c + j) == tgt ? 1.f : 0.f)) * gs;
      }
      store8(z + c, f);
    } else {
      for (int j = 0; j < 8 && c + j < V; ++j) {
        float p = __expf(bf16_to_f32(z[c + j]) - rmax) * inv;
        z[c + j] = f32_to_bf16((p - ((c + j) == tgt ? 1.f : 0.f)) * gs);
      }
    }
  }
}

// Single-read variant: the whole row is staged in shared memory (V*2 bytes)
// while the online max/sum runs, so the logits are read from HBM once.
__global__ void __launch_bounds__(kXentThreads) xent_smem_kernel(__nv_bfloat16* __restrict__ logits,
                                                                 const int64_t* __restrict__ targets,
                                                                 float* __restrict__ loss, int V, long long ld,
                                                                 float grad_scale, int ignore_index) {
  extern __shared__ __align__(16) uint8_t xs_raw[];
  __nv_bfloat16* row_s = reinterpret_cast<__nv_bfloat16*>(xs_raw);
  __shared__ float sm[32], ss[32];
  __shared__ __align__(8) uint64_t bar;
  const int row = blockIdx.x;
  __nv_bfloat16* z = logits + static_cast<long long>(row) * ld;
  // One bulk (TMA) copy brings the whole row in: far more bytes in flight per
  // SM than per-thread loads, which is what a streaming kernel needs.
  const uint32_t bar_a = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(bar_a, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t bytes = static_cast<uint32_t>(V) * 2;
    mbar_arrive_expect_tx(bar_a, bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(row_s)), "l"(z), "r"(bytes), "r"(bar_a) : "memory");
  }
  mbar_wait(bar_a, 0, nullptr);
  // Three passes over the row in shared memory, one exponential per element:
  // max; e = exp(z - max) with its sum (e written back over the logits, bf16 --
  // the gradient is rounded to bf16 anyway); gradient = e / sum - onehot.
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t tgt = targets[row];
  const bool ignored = tgt == ignore_index;
  const float z_tgt = ignored ? 0.f : bf16_to_f32(row_s[tgt]);  // read before pass 2 overwrites it
  float m = -INFINITY;
  for (int c = threadIdx.x * 8; c < V; c += kXentThreads * 8) {
    float f[8];
    load8(row_s + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, f[j]);
  }
  m = warp_max(m);
  if (lane == 0) sm[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = warp_max(lane < kXentThreads / 32 ? sm[lane] : -INFINITY);
    if (lane == 0) sm[0] = m;
  }
  __syncthreads();
  const float rmax = sm[0];
  float s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += kXentThreads * 8) {
    float f[8];
    load8(row_s + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      f[j] = __expf(f[j] - rmax);
      s += f[j];
    }
    store8(row_s + c, f);
  }
  s = warp_sum(s);
  if (lane == 0) ss[warp] = s;
  __syncthreads();
  if (warp == 0) {
    s = warp_sum(lane < kXentThreads / 32 ? ss[lane] : 0.f);
    if (lane == 0) ss[0] = s;
  }
  __syncthreads();
  const float inv = 1.f / ss[0];
  if (threadIdx.x == 0) loss[row] = ignored ? 0.f : (rmax + logf(ss[0]) - z_tgt);
  const float gs = ignored ? 0.f : grad_scale;
  for (int c = threadIdx.x * 8; c < V; c += kXentThreads * 8) {
    float f[8];
    load8(row_s + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = (f[j] * inv - ((c + j) == tgt ? 1.f : 0.f)) * gs;
    store8(z + c, f);
  }
}

// ---------------------------------------------------------------------------
// Multi-tensor AdamW with fp32 master weights.
//   table rows: {param(bf16 or fp32), grad(bf16 or fp32), master(fp32 or null), m, v, numel}
// ---------------------------------------------------------------------------
struct AdamEntry {
  void* param;
  const void* grad;
  float* master;
  float* m;
  float* v;
  long long numel;
};

struct AdamChunk {
  long long entry;
  long long start;
  long long len;
};

// One chunk (<= 64K contiguous elements of one tensor) per block iteration:
// no per-element search, fully coalesced accesses.
__global__ void __launch_bounds__(512) adamw_kernel(const AdamEntry* __restrict__ table,
                                                    const AdamChunk* __restrict__ chunks, int n_chunks,
                                                    int param_bf16, int grad_bf16, float lr, float beta1, float beta2,
                                                    float eps, float wd, float bc1, float bc2, float grad_scale) {
  const float c1 = 1.f / bc1;
  const float c2 = 1.f / bc2;
  for (int ci = blockIdx.x; ci < n_chunks; ci += gridDim.x) {
    const AdamChunk ch = chunks[ci];
    const AdamEntry e = table[ch.entry];
    const long long end = ch.start + ch.len;
    // 4 elements per thread when every stream of this chunk is 16-byte (fp32) / 8-byte (bf16) aligned
    const uintptr_t al = reinterpret_cast<uintptr_t>(e.m) | reinterpret_cast<uintptr_t>(e.v) |
                         reinterpret_cast<uintptr_t>(e.master) |
                         (reinterpret_cast<uintptr_t>(e.param) << (param_bf16 ? 1 : 0)) |
                         (reinterpret_cast<uintptr_t>(e.grad) << (grad_bf16 ? 1 : 0));
    if ((al & 15) == 0 && ch.start % 4 == 0 && ch.len % 4 == 0) {
      for (long long k = ch.start + 4 * threadIdx.x; k < end; k += 4 * blockDim.x) {
        float g[4], w[4];
        if (grad_bf16) {
          const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(e.grad) + k);
          const float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
          g[0] = a.x; g[1] = a.y; g[2] = b.x; g[3] = b.y;
        } else {
          const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(e.grad) + k);
          g[0] = f.x; g[1] = f.y; g[2] = f.z; g[3] = f.w;
        }
        if (e.master) {
          const float4 f = *reinterpret_cast<const float4*>(e.master + k);
          w[0] = f.x; w[1] = f.y; w[2] = f.z; w[3] = f.w;
        } else if (param_bf16) {
          const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(e.param) + k);
          const float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
          w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y;
        } else {
          const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(e.param) + k);
          w[0] = f.x; w[1] = f.y; w[2] = f.z; w[3] = f.w;
        }
        const float4 m4 = *reinterpret_cast<const float4*>(e.m + k), v4 = *reinterpret_cast<const float4*>(e.v + k);
        float m[4] = {m4.x, m4.y, m4.z, m4.w}, v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          g[i] *= grad_scale;
          m[i] = beta1 * m[i] + (1.f - beta1) * g[i];
          v[i] = beta2 * v[i] + (1.f - beta2) * g[i] * g[i];
          w[i] -= lr * wd * w[i];
          w[i] -= lr * (m[i] * c1) / (sqrtf(v[i] * c2) + eps);
        }
        *reinterpret_cast<float4*>(e.m + k) = make_float4(m[0], m[1], m[2], m[3]);
        *reinterpret_cast<float4*>(e.v + k) = make_float4(v[0], v[1], v[2], v[3]);
        if (e.master) *reinterpret_cast<float4*>(e.master + k) = make_float4(w[0], w[1], w[2], w[3]);
        if (param_bf16)
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(e.param) + k) =
              make_uint2(pack_bf16x2(w[0], w[1]), pack_bf16x2(w[2], w[3]));
        else
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(e.param) + k) = make_float4(w[0], w[1], w[2], w[3]);
      }
      continue;
    }
    for (long long k = ch.start + threadIdx.x; k < end; k += blockDim.x) {
      float g = grad_bf16 ? bf16_to_f32(reinterpret_cast<const __nv_bfloat16*>(e.grad)[k])
                          : reinterpret_cast<const float*>(e.grad)[k];
      g *= grad_scale;
      float w = e.master ? e.master[k]
                         : (param_bf16 ? bf16_to_f32(reinterpret_cast<__nv_bfloat16*>(e.param)[k])
                                       : reinterpret_cast<float*>(e.param)[k]);
      const float m = beta1 * e.m[k] + (1.f - beta1) * g;
      const float v = beta2 * e.v[k] + (1.f - beta2) * g * g;
      e.m[k] = m;
      e.v[k] = v;
      w -= lr * wd * w;
      w -= lr * (m * c1) / (sqrtf(v * c2) + eps);
      if (e.master) e.master[k] = w;
      if (param_bf16) reinterpret_cast<__nv_bfloat16*>(e.param)[k] = f32_to_bf16(w);
      else reinterpret_cast<float*>(e.param)[k] = w;
    }
  }
}

// ---------------------------------------------------------------------------
// host wrappers
// ---------------------------------------------------------------------------
static void check_bf16(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), n,
              " must be a contiguous CUDA bf16 tensor");
}

// Resident blocks per SM x SMs of `kern` at this block size and dynamic shared
// memory (the one-wave grid of the grid-stride kernels), with the shared-memory
// opt-in applied: queried once per (kernel, device, smem) instead of per call.
static int resident_wave(const void* kern, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t>, int> cache;
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(kern, dev, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (smem > 48 * 1024)
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  int per_sm = 1, sms = 148;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem));
  const int wave = std::max(1, per_sm) * sms;
  cache.emplace(key, wave);
  return wave;
}

void layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, torch::Tensor y, torch::Tensor mean,
                   torch::Tensor rstd, double eps) {
  check_bf16(x, "x");
  check_bf16(w, "weight");
  check_bf16(b, "bias");
  check_bf16(y, "y");
  const int C = static_cast<int>(x.size(-1));
  TORCH_CHECK(C % 8 == 0, "LayerNorm width must be a multiple of 8");
  const int rows = static_cast<int>(x.numel() / C);
  c10::cuda::CUDAGuard g(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  const auto* bp = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  const float e = static_cast<float>(eps);
  // grid-stride kernels: one wave of resident blocks (w and b are loaded once per warp)
  auto wave_of = [&](auto kern) {
    return std::max(1, std::min((rows + 7) / 8, resident_wave(reinterpret_cast<const void*>(kern), 256, 0)));
  };
  auto reg = [&](auto kern) {
    kern<<<wave_of(kern), 256, 0, stream>>>(xp, wp, bp, yp, mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, e);
  };
  if (C == 256) reg(layernorm_fwd_reg_kernel<1>);
  else if (C == 512) reg(layernorm_fwd_reg_kernel<2>);
  else if (C == 768) reg(layernorm_fwd_reg_kernel<3>);
  else if (C == 1024) reg(layernorm_fwd_reg_kernel<4>);
  else if (C % 256 == 0 && C >= 1536 && C <= 4096)
    layernorm_fwd_wide_kernel<<<std::max(1, std::min(148 * 4, rows)), C / 8, 0, stream>>>(
        xp, wp, bp, yp, mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, C, e);
  else
    layernorm_fwd_kernel<<<(rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0, stream>>>(
        xp, wp, bp, yp, mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, C, e);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// A fold launch that fails leaves its accumulator in an unknown state (the
// partial sums and arrival counter of blocks that ran); every later fold of
// that size would carry them.  Clear it before reporting the error.
static void check_fold_launch(const torch::Tensor& acc, int64_t n_values, cudaStream_t stream) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return;
  cudaMemsetAsync(acc.data_ptr(), 0, static_cast<size_t>(n_values + 1) * sizeof(float), stream);
  TORCH_CHECK(false, "column-sum fold launch failed (accumulator cleared): ", cudaGetErrorString(e));
}

int ln_bwd_blocks(int rows) { return std::max(1, std::min(148 * 2, (rows + kRowWarps - 1) / kRowWarps)); }

static void layernorm_bwd_impl(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                               torch::Tensor rstd, torch::Tensor dx, torch::Tensor dw, torch::Tensor db,
                               torch::Tensor partials, bool accumulate, const torch::Tensor* add) {
  check_bf16(dy, "dy");
  check_bf16(x, "x");
  check_bf16(dx, "dx");
  const int C = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / C);
  const int blocks = ln_bwd_blocks(rows);
  TORCH_CHECK(partials.numel() >= 2LL * C + 1 && partials.scalar_type() == at::kFloat,
              "the fold accumulator must hold 2C + 1 floats (zeroed, persistent)");
  c10::cuda::CUDAGuard g(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const size_t smem = 2 * C * sizeof(float);
  const bool f32 = dw.scalar_type() == at::kFloat;
  auto launch = [&](auto kern) {
    // one wave: as many blocks as can be resident (these kernels grid-stride over rows)
    const int wave =
        std::max(1, std::min(blocks, resident_wave(reinterpret_cast<const void*>(kern), kRowWarps * 32, smem)));
    kern<<<wave, kRowWarps * 32, smem, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), partials.data_ptr<float>(), rows, C, dw.data_ptr(),
        db.data_ptr(), f32 ? 1 : 0, accumulate ? 1 : 0);
  };
  // rows reach shared memory by bulk copies: 16-byte aligned row starts needed
  const bool bulk = reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(dy.data_ptr()) % 16 == 0 && x.is_contiguous() && dy.is_contiguous() &&
                    (add == nullptr || (add->is_contiguous() && reinterpret_cast<uintptr_t>(add->data_ptr()) % 16 == 0));
  const __nv_bfloat16* add_p = add ? reinterpret_cast<const __nv_bfloat16*>(add->data_ptr()) : nullptr;
  auto launch_bulk = [&](auto kern, size_t bytes) {
    const int wave =
        std::max(1, std::min(blocks, resident_wave(reinterpret_cast<const void*>(kern), kRowWarps * 32, bytes)));
    kern<<<wave, kRowWarps * 32, bytes, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), partials.data_ptr<float>(), rows, C, dw.data_ptr(),
        db.data_ptr(), f32 ? 1 : 0, accumulate ? 1 : 0, add_p);
  };
  if (add != nullptr && bulk && C == 256) launch_bulk(layernorm_bwd_bulk_kernel<1, 8, true>, ln_bwd_bulk_smem<1, 8, true>());
  else if (add != nullptr && bulk && C == 512) launch_bulk(layernorm_bwd_bulk_kernel<2, 8, true>, ln_bwd_bulk_smem<2, 8, true>());
  else if (add != nullptr && bulk && C == 768) launch_bulk(layernorm_bwd_bulk_kernel<3, 5, true>, ln_bwd_bulk_smem<3, 5, true>());
  else if (add != nullptr && bulk && C == 1024) launch_bulk(layernorm_bwd_bulk_kernel<4, 3, true>, ln_bwd_bulk_smem<4, 3, true>());
  else if (bulk && C == 256) launch_bulk(layernorm_bwd_bulk_kernel<1, 8>, ln_bwd_bulk_smem<1, 8>());
  else if (bulk && C == 512) launch_bulk(layernorm_bwd_bulk_kernel<2, 8>, ln_bwd_bulk_smem<2, 8>());
  else if (bulk && C == 768) launch_bulk(layernorm_bwd_bulk_kernel<3, 6>, ln_bwd_bulk_smem<3, 6>());
  else if (bulk && C == 1024) launch_bulk(layernorm_bwd_bulk_kernel<4, 4>, ln_bwd_bulk_smem<4, 4>());
  else if (C == 256) launch(layernorm_bwd_kernel<1>);
  else if (C == 512) launch(layernorm_bwd_kernel<2>);
  else if (C == 768) launch(layernorm_bwd_kernel<3>);
  else if (C == 1024) launch(layernorm_bwd_kernel<4>);
  else if (C % 256 == 0 && C >= 1536 && C <= 4096)
    layernorm_bwd_wide_kernel<<<blocks, C / 8, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), partials.data_ptr<float>(), rows, C, dw.data_ptr(),
        db.data_ptr(), f32 ? 1 : 0, accumulate ? 1 : 0);
  else launch(layernorm_bwd_kernel<0>);
  check_fold_launch(partials, 2LL * C, stream);
  const bool fused = add != nullptr && bulk && (C == 256 || C == 512 || C == 768 || C == 1024);
  if (add != nullptr && !fused) dx.add_(*add);
}

void layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean, torch::Tensor rstd,
                   torch::Tensor dx, torch::Tensor dw, torch::Tensor db, torch::Tensor partials, bool accumulate) {
  layernorm_bwd_impl(dy, x, w, mean, rstd, dx, dw, db, partials, accumulate, nullptr);
}

// dx = LayerNorm backward + add (the gradient x also receives through a
// residual branch), dgamma / dbeta as layernorm_bwd.
void layernorm_bwd_add(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean, torch::Tensor rstd,
                       torch::Tensor add, torch::Tensor dx, torch::Tensor dw, torch::Tensor db, torch::Tensor partials,
                       bool accumulate) {
  check_bf16(add, "add");
  TORCH_CHECK(add.numel() == x.numel(), "add must match x");
  layernorm_bwd_impl(dy, x, w, mean, rstd, dx, dw, db, partials, accumulate, &add);
}

// Bias gradient in one kernel: column sums of a 128-row band per block,
// added into the persistent accumulator, finished by the last block.
__global__ void __launch_bounds__(256) colsum_fold_kernel(const __nv_bfloat16* __restrict__ g, float* acc, int rows,
                                                          int C, void* out, int out_f32, int accumulate) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * kColRows;
  const int r1 = min(rows, r0 + kColRows);
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c0 < C) {
    // all of this warp's kColRows / 8 rows in flight at once (16 x 16 B per
    // lane): one warp's loads cover the HBM latency instead of four
    constexpr int kPer = kColRows / 8;
    uint4 raw[kPer];
    const __nv_bfloat16* p = g + static_cast<long long>(r0 + warp) * C + c0;
    if (r1 - r0 == kColRows) {  // full band: unconditional loads, all issued before the first add
#pragma unroll
      for (int i = 0; i < kPer; ++i) raw[i] = ld_v4(p + static_cast<long long>(8 * i) * C);
    } else {
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        raw[i] = r0 + warp + 8 * i < r1 ? ld_v4(p + static_cast<long long>(8 * i) * C) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const uint32_t ws[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(ws[j]);
        s[2 * j] += f.x;
        s[2 * j + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = s[j];
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < C) atomicAdd(acc + c, t);
  finish_fold(acc, C, out, out, C, out_f32, accumulate);
}

int colsum_row_blocks(int rows) { return std::max(1, (rows + kColRows - 1) / kColRows); }

void bias_grad(torch::Tensor g, torch::Tensor out, torch::Tensor partials, bool accumulate) {
  check_bf16(g, "grad");
  const int C = static_cast<int>(g.size(-1));
  TORCH_CHECK(C % 8 == 0, "bias width must be a multiple of 8");
  const int rows = static_cast<int>(g.numel() / C);
  const int yb = colsum_row_blocks(rows);
  TORCH_CHECK(partials.numel() >= static_cast<int64_t>(C) + 1 && partials.scalar_type() == at::kFloat,
              "the fold accumulator must hold C + 1 floats (zeroed, persistent)");
  c10::cuda::CUDAGuard guard(g.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  colsum_fold_kernel<<<dim3((C + 255) / 256, yb), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), partials.data_ptr<float>(), rows, C, out.data_ptr(),
      out.scalar_type() == at::kFloat ? 1 : 0, accumulate ? 1 : 0);
  check_fold_launch(partials, C, stream);
}

static int elementwise_blocks(long long n8) {
  return static_cast<int>(std::max(1LL, std::min((n8 + 255) / 256, 148LL * 16)));
}

void gelu_fwd(torch::Tensor x, torch::Tensor y) {
  check_bf16(x, "x");
  TORCH_CHECK(x.numel() % 8 == 0, "numel must be a multiple of 8");
  const long long n8 = x.numel() / 8;
  c10::cuda::CUDAGuard g(x.device());
  gelu_fwd_kernel<<<elementwise_blocks(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_bwd(torch::Tensor x, torch::Tensor dy, torch::Tensor dx) {
  check_bf16(x, "x");
  const long long n8 = x.numel() / 8;
  c10::cuda::CUDAGuard g(x.device());
  gelu_bwd_kernel<<<elementwise_blocks(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_fwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor wpe, torch::Tensor y) {
  check_bf16(wte, "wte");
  check_bf16(wpe, "wpe");
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous(), "idx must be int64");
  const int T = static_cast<int>(idx.size(-1));
  const int C = static_cast<int>(wte.size(1));
  const int tokens = static_cast<int>(idx.numel());
  c10::cuda::CUDAGuard g(wte.device());
  embed_fwd_kernel<<<(tokens + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(wte.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(wpe.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), tokens,
      T, C);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_bwd(torch::Tensor idx, torch::Tensor dy, torch::Tensor dwte, torch::Tensor dwpe, bool accumulate_pos) {
  check_bf16(dy, "dy");
  const int B = static_cast<int>(idx.size(0));
  const int T = static_cast<int>(idx.size(1));
  const int C = static_cast<int>(dwte.size(1));
  const int tokens = B * T;
  c10::cuda::CUDAGuard g(dy.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  embed_bwd_tok_kernel<<<(tokens + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0, stream>>>(
      idx.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dwte.data_ptr()), tokens, C);
  embed_bwd_pos_kernel<<<T, 128, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                                             reinterpret_cast<__nv_bfloat16*>(dwpe.data_ptr()), B, T, C,
                                             accumulate_pos ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void xent_fwd_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss, double grad_scale,
                  int64_t ignore_index) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1,
              "logits must be row-major bf16");
  TORCH_CHECK(targets.scalar_type() == at::kLong, "targets must be int64");
  const int rows = static_cast<int>(logits.size(0));
  const int V = static_cast<int>(logits.size(1));
  TORCH_CHECK(logits.stride(0) % 8 == 0, "logits row stride must be a multiple of 8");
  c10::cuda::CUDAGuard g(logits.device());
  const size_t row_bytes = static_cast<size_t>(V) * 2;
  if (V % 8 == 0 && row_bytes <= 200 * 1024 && (logits.stride(0) * 2) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0) {
    static size_t configured = 0;
    if (row_bytes > configured) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(xent_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(row_bytes)));
      configured = row_bytes;
    }
    xent_smem_kernel<<<rows, kXentThreads, row_bytes, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), loss.data_ptr<float>(), V,
        logits.stride(0), static_cast<float>(grad_scale), static_cast<int>(ignore_index));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  xent_fwd_bwd_kernel<<<rows, kXentThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), loss.data_ptr<float>(), V,
      logits.stride(0), static_cast<float>(grad_scale), static_cast<int>(ignore_index));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// table: int64 [n, 6] {param, grad, master, m, v, numel}; chunks: int64 [c, 3] {entry, start, len}.
void adamw_step(torch::Tensor table, torch::Tensor chunks, bool param_bf16, bool grad_bf16, double lr, double beta1,
                double beta2, double eps, double wd, double bc1, double bc2, double grad_scale) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kLong && table.size(1) == 6, "bad AdamW table");
  TORCH_CHECK(chunks.is_cuda() && chunks.scalar_type() == at::kLong && chunks.size(1) == 3, "bad AdamW chunks");
  c10::cuda::CUDAGuard g(table.device());
  const int n_chunks = static_cast<int>(chunks.size(0));
  const int blocks = std::max(1, std::min(n_chunks, 148 * 8));
  adamw_kernel<<<blocks, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const AdamEntry*>(table.data_ptr()), reinterpret_cast<const AdamChunk*>(chunks.data_ptr()),
      n_chunks, param_bf16, grad_bf16, static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2),
      static_cast<float>(eps), static_cast<float>(wd), static_cast<float>(bc1), static_cast<float>(bc2),
      static_cast<float>(grad_scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mnb

namespace mnb {

// One %globaltimer reading (ns) into out[idx], in stream order: places host-
// side events (a DDP bucket becoming ready, the end of backward) on the same
// clock as the device event ring's collective start / end stamps.
__global__ void stamp_kernel(unsigned long long* out, int idx) {
  if (threadIdx.x == 0) out[idx] = globaltimer_ns();
}

void stamp(torch::Tensor out, int64_t idx) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kLong && idx >= 0 && idx < out.numel(),
              "stamp: int64 CUDA tensor and an index inside it");
  stamp_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<unsigned long long*>(out.data_ptr()), static_cast<int>(idx));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mnb
