// Device communicator: collectives as single kernels over NVLink peer memory.
//
// Runtime (host):
//   * every rank cudaMallocs a staging buffer and a signal pad, exports both
//     with cudaIpcGetMemHandle; the Python layer all-gathers the handles over
//     the host transport and each rank opens its peers' (lazy peer access), so
//     kernels can dereference every peer's memory directly;
//   * further "symmetric segments" (DDP gradient buckets, FSDP shards) are
//     exported/opened the same way, so collectives on them need no copy-in;
//   * a status block and a ring of kernel-level event records live in
//     host-mapped pinned memory: kernels write them, the host reads them
//     without synchronising (timeouts, flight recorder).
//
// Kernels (sm_100a, no tensor cores needed -- these are bandwidth kernels):
//   one_shot   every rank reads all W inputs, reduces in a fixed rank order
//              (bitwise-identical results everywhere); latency-optimal.
//   two_shot   reduce-scatter (rank r reduces its 1/W) then all-gather of the
//              reduced chunks; bandwidth-optimal on NVSwitch.  Works in place
//              on a symmetric buffer (the DDP bucket path).
//   reduce_scatter / all_gather / broadcast / all_to_all / barrier
//   stepped    cooperative executor for the ring / tree / halving / naive
//              schedules (per-hop wire rounding reproduces the host path's
//              numerics), one grid-wide sync plus one cross-rank barrier per
//              schedule step.
// Every kernel accumulates in fp32 (int64 for integers), applies an optional
// scale (1/W for averaging) before the single final rounding, and can carry
// a narrower wire type (bf16) than its input/output (fp32).
//
// Synchronisation: per (block, source rank) signal slots holding monotonically
// increasing epochs.  A block publishes with __syncthreads + system fence +
// st.release.sys into each peer's slot and waits with ld.acquire.sys on its
// own slots.  Each wait polls %globaltimer against a deadline; on expiry it
// records {code, peer, block, seq} in the status block and the kernel
// returns.  Nothing traps, nothing spins unbounded.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "nvls.h"
#include "peer.cuh"

namespace cg = cooperative_groups;

namespace mnb {

constexpr int kCommThreads = 512;
constexpr int kRingCap = 4096;

enum OpCode : int { kSum = 0, kProd = 1, kMax = 2, kMin = 3 };

struct DevEvent {
  uint32_t seq;
  int32_t op;
  int64_t nbytes;
  uint64_t t_start;
  uint64_t t_end;
  int32_t status;
  int32_t pad;
};

struct CommArgs {
  void* data[kMaxRanks];     // per-rank peer-visible staging region for this call
  void* dst[kMaxRanks];      // per-rank symmetric output (in-place all-reduce), or null
  uint32_t* sig[kMaxRanks];  // per-rank signal pads
  const void* in;
  void* out;
  long long n;      // elements (all_reduce / broadcast) or per-rank chunk (rs/ag/a2a)
  int rank, world, root;
  uint32_t epoch;
  float scale;
  int copy_in;
  volatile int* status;  // host-mapped [4]
  unsigned long long timeout_ns;
  DevEvent* ring;        // host-mapped [kRingCap]
  uint32_t seq;
  int opname;
  long long nbytes;
};

// ---------------------------------------------------------------------------
// barrier among the block-`b` CTAs of every rank
// ---------------------------------------------------------------------------
MNB_DEVICE bool peer_barrier(const CommArgs& a, uint32_t value) {
  const int b = blockIdx.x;
  __syncthreads();
  const int t = threadIdx.x;
  if (t < a.world && t != a.rank) {
    __threadfence_system();
    st_release_sys(a.sig[t] + b * kMaxRanks + a.rank, value);
  }
  bool ok = true;
  if (t < a.world && t != a.rank) {
    const uint32_t* slot = a.sig[a.rank] + b * kMaxRanks + t;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (static_cast<int32_t>(ld_acquire_sys(slot) - value) < 0) {
      if ((++spins & 255u) == 0) {
        if (a.status[0] != 0) { ok = false; break; }
        if (globaltimer_ns() - t0 > a.timeout_ns) {
          if (a.status[0] == 0) {
            a.status[1] = t;
            a.status[2] = b;
            a.status[3] = static_cast<int>(a.seq);
            __threadfence_system();
            a.status[0] = kErrPeerTimeout;
          }
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

MNB_DEVICE void ring_begin(const CommArgs& a) {
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.ring != nullptr) {
    DevEvent* e = a.ring + (a.seq % kRingCap);
    e->t_end = 0;
    e->status = -1;
    e->op = a.opname;
    e->nbytes = a.nbytes;
    e->t_start = globaltimer_ns();
    __threadfence_system();
    e->seq = a.seq;
  }
}
MNB_DEVICE void ring_end(const CommArgs& a, bool ok) {
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.ring != nullptr) {
    DevEvent* e = a.ring + (a.seq % kRingCap);
    e->status = ok ? 0 : a.status[0];
    __threadfence_system();
    e->t_end = globaltimer_ns();
  }
}

// ---------------------------------------------------------------------------
// element conversion helpers
// ---------------------------------------------------------------------------
template <typename T> MNB_DEVICE float to_f(T x);
template <> MNB_DEVICE float to_f<float>(float x) { return x; }
template <> MNB_DEVICE float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> MNB_DEVICE float to_f<__half>(__half x) { return __half2float(x); }
template <typename T> MNB_DEVICE T from_f(float x);
template <> MNB_DEVICE float from_f<float>(float x) { return x; }
template <> MNB_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> MNB_DEVICE __half from_f<__half>(float x) { return __float2half_rn(x); }

template <typename T> struct Acc { using type = float; };
template <> struct Acc<int64_t> { using type = long long; };
template <> struct Acc<int32_t> { using type = long long; };

template <typename TA, typename T> MNB_DEVICE TA widen(T x) { return static_cast<TA>(to_f<T>(x)); }
template <> MNB_DEVICE long long widen<long long, int64_t>(int64_t x) { return x; }
template <> MNB_DEVICE long long widen<long long, int32_t>(int32_t x) { return x; }
template <typename T, typename TA> MNB_DEVICE T narrow(TA x) { return from_f<T>(static_cast<float>(x)); }
template <> MNB_DEVICE int64_t narrow<int64_t, long long>(long long x) { return x; }
template <> MNB_DEVICE int32_t narrow<int32_t, long long>(long long x) { return static_cast<int32_t>(x); }

template <int OP, typename TA> MNB_DEVICE TA combine(TA a, TA b) {
  if (OP == kSum) return a + b;
  if (OP == kProd) return a * b;
  if (OP == kMax) return a > b ? a : b;
  return a < b ? a : b;
}

template <int OP, typename TA> MNB_DEVICE TA finish(TA x, float scale) {
  if (OP == kSum && scale != 1.0f) return static_cast<TA>(static_cast<float>(x) * scale);
  return x;
}

// VEC wire elements per 16-byte access.
template <typename TW> struct Vec { static constexpr int n = 16 / sizeof(TW); };

template <typename TW, typename TA>
MNB_DEVICE void load_vec(const void* p, TA* v) {
  uint4 raw = ld_v4_volatile(p);
  const TW* e = reinterpret_cast<const TW*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<TW>::n; ++i) v[i] = widen<TA, TW>(e[i]);
}
template <typename TW, typename TA>
MNB_DEVICE void store_vec(void* p, const TA* v) {
  uint4 raw;
  TW* e = reinterpret_cast<TW*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<TW>::n; ++i) e[i] = narrow<TW, TA>(v[i]);
  st_v4(p, raw);
}
// Store VEC values as the (possibly wider) output type.
template <typename TO, typename TA, int N>
MNB_DEVICE void store_out(TO* p, const TA* v) {
#pragma unroll
  for (int i = 0; i < N; ++i) p[i] = narrow<TO, TA>(v[i]);
}

// Block-range of [0, n) for this CTA.
MNB_DEVICE void block_range(long long n, long long* lo, long long* hi) {
  const long long per = (n + gridDim.x - 1) / gridDim.x;
  *lo = min(n, per * blockIdx.x);
  *hi = min(n, *lo + per);
}

// Stage [lo, hi) units of the local input into this rank's wire buffer.
template <typename TI, typename TW>
MNB_DEVICE void copy_in_units(const CommArgs& a, long long lo, long long hi) {
  constexpr int V = Vec<TW>::n;
  using TA = typename Acc<TW>::type;
  const TI* in = reinterpret_cast<const TI*>(a.in);
  TW* w = reinterpret_cast<TW*>(a.data[a.rank]);
  for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
    TA v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = widen<TA, TI>(in[u * V + i]);
    store_vec<TW, TA>(w + u * V, v);
  }
}

// L2-only 16-byte load (bypasses L1: staging is rewritten by peers every call).
MNB_DEVICE uint4 ld_v4_cg(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
template <typename TW, typename TA>
MNB_DEVICE void unpack_vec(uint4 raw, TA* v) {
  const TW* e = reinterpret_cast<const TW*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<TW>::n; ++i) v[i] = widen<TA, TW>(e[i]);
}
template <typename TW, typename TA>
MNB_DEVICE uint4 pack_vec(const TA* v) {
  uint4 raw;
  TW* e = reinterpret_cast<TW*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<TW>::n; ++i) e[i] = narrow<TW, TA>(v[i]);
  return raw;
}
// One VEC of the (possibly wider) input, converted to the accumulation type.
template <typename TI, typename TA, int V>
MNB_DEVICE void load_in(const TI* p, TA* v) {
  if constexpr (sizeof(TI) * V == 16) {
    uint4 raw = ld_v4(p);
    const TI* e = reinterpret_cast<const TI*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = widen<TA, TI>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = widen<TA, TI>(p[i]);
  }
}
template <typename T>
MNB_DEVICE T* at(void* base, long long elems) {
  return reinterpret_cast<T*>(base) + elems;
}

// ---------------------------------------------------------------------------
// all-reduce, one shot, push (latency path, small messages)
//   staging (wire type): [parity 2][W slots][n_pad].  Every rank stores its
//   whole input into slot `rank` of every peer (posted NVLink writes), one
//   barrier, then every rank reduces its W local slots in rank order, so all
//   ranks produce identical bits.  Calls alternate the parity half so a fast
//   peer's next call never overwrites slots still being reduced here.
// ---------------------------------------------------------------------------
template <typename TI, typename TW, int OP>
__global__ void __launch_bounds__(kCommThreads) ar_push_one_shot_kernel(CommArgs a, long long n_pad) {
  using TA = typename Acc<TW>::type;
  constexpr int V = Vec<TW>::n;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long nu = a.n / V, tail = a.n - nu * V;
  const long long par = 0;  // the host already selected this call's staging half
  long long lo, hi;
  block_range(nu, &lo, &hi);
  const TI* in = reinterpret_cast<const TI*>(a.in);
  for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
    TA v[V];
    load_in<TI, TA, V>(in + u * V, v);
    const uint4 w = pack_vec<TW, TA>(v);
    for (int k = 1; k < W; ++k) {
      const int p = (r + k) % W;
      st_v4(at<TW>(a.data[p], par + r * n_pad + u * V), w);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < tail) {
    const TW w = narrow<TW, TA>(widen<TA, TI>(in[nu * V + threadIdx.x]));
    for (int p = 0; p < W; ++p) *at<TW>(a.data[p], par + r * n_pad + nu * V + threadIdx.x) = w;
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  if (ok) {
    TI* out = reinterpret_cast<TI*>(a.out);
    for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
      TA acc[V], v[V];
      for (int p = 0; p < W; ++p) {  // rank order on every rank: identical bits everywhere
        if (p == r) {
          load_in<TI, TA, V>(in + u * V, v);
#pragma unroll
          for (int i = 0; i < V; ++i) v[i] = widen<TA, TW>(narrow<TW, TA>(v[i]));
        } else {
          unpack_vec<TW, TA>(ld_v4_cg(at<TW>(a.data[r], par + p * n_pad + u * V)), v);
        }
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = p == 0 ? v[i] : combine<OP>(acc[i], v[i]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc[i], a.scale)));
      store_out<TI, TA, V>(out + u * V, acc);
    }
    if (blockIdx.x == 0 && threadIdx.x < tail) {
      const long long e = nu * V + threadIdx.x;
      TA acc = widen<TA, TW>(*reinterpret_cast<volatile TW*>(at<TW>(a.data[r], par + e)));
      for (int p = 1; p < W; ++p)
        acc = combine<OP>(acc, widen<TA, TW>(*reinterpret_cast<volatile TW*>(at<TW>(a.data[r], par + p * n_pad + e))));
      out[e] = narrow<TI, TA>(widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc, a.scale))));
    }
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// all-reduce, two shot, push (bandwidth path)
//   staging (wire type): [W slots][chunk] | [W][chunk] results | [W][V] tail
//   phase 1  rank r stores chunk c of its input into slot r of rank c
//   phase 2  rank r reduces its W slots (local reads, rank order), scales,
//            and stores the result into chunk r of every rank: straight into
//            their tensors when those are symmetric (DDP buckets, in place),
//            else into their result region
//   phase 3  (non-symmetric) copy the other ranks' chunks out of the result
//            region.
//   Every element is reduced once, by its owner, so all ranks hold
//   identical bits.  Two barriers; no trailing one is needed because a
//   peer's next phase-1 writes wait for this rank's phase-2 signal.
// ---------------------------------------------------------------------------
// THREADS / MINB: the default is 512-thread CTAs.  The "beside compute"
// variant (128 threads, at most 80 registers) leaves room on an SM for one CTA
// of the persistent tcgen05 GEMM / attention kernels (320 threads x 168
// registers): comm CTAs that need a whole SM would keep those kernels' CTAs
// from starting, and each such CTA's fixed share of tiles would then finish
// late (DDP runs this kernel during the backward pass).
template <typename TI, typename TW, int OP, int THREADS = kCommThreads, int MINB = 1>
__global__ void __launch_bounds__(THREADS, MINB) ar_push_two_shot_kernel(CommArgs a, long long chunk_u) {
  using TA = typename Acc<TW>::type;
  constexpr int V = Vec<TW>::n;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long nu = a.n / V, tail = a.n - nu * V;
  const long long cw = chunk_u * V;                   // chunk length in elements
  const long long res_off = W * cw, tail_off = 2 * W * cw;
  const long long sub = (chunk_u + gridDim.x - 1) / gridDim.x;
  auto sub_range = [&](int c, long long* lo, long long* hi) {
    const long long c0 = min(nu, c * chunk_u), c1 = min(nu, c0 + chunk_u);
    *lo = min(c1, c0 + sub * blockIdx.x);
    *hi = min(c1, *lo + sub);
  };
  const bool sym = a.dst[r] != nullptr;
  const TI* in = reinterpret_cast<const TI*>(a.in);
  // phase 1: scatter my chunks into their owners' slot r (my own chunk stays
  // in my input; phase 2 reads it from there)
  for (int k = 1; k < W; ++k) {
    const int c = (r + k) % W;
    long long lo, hi;
    sub_range(c, &lo, &hi);
    constexpr int U = 4;  // independent 16-byte loads in flight per thread before the stores
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
      uint4 w[U];
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const long long u = u0 + j * blockDim.x;
        if (u < hi) {
          TA v[V];
          load_in<TI, TA, V>(in + u * V, v);
          w[j] = pack_vec<TW, TA>(v);
        }
      }
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const long long u = u0 + j * blockDim.x;
        if (u < hi) st_v4(at<TW>(a.data[c], r * cw + (u - c * chunk_u) * V), w[j]);
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < tail) {
    const TW w = narrow<TW, TA>(widen<TA, TI>(in[nu * V + threadIdx.x]));
    for (int p = 0; p < W; ++p) *at<TW>(a.data[p], tail_off + r * V + threadIdx.x) = w;
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  TI* out = reinterpret_cast<TI*>(a.out);
  if (ok) {
    long long lo, hi;
    sub_range(r, &lo, &hi);
    // units per thread per pass: U2 independent loads per source rank (2 in
    // the small-CTA variant, whose 80-register budget holds U2 x V accumulators)
    constexpr int U2 = THREADS >= 512 ? 4 : 2;
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U2 * blockDim.x) {
      TA accs[U2][V];
      // rank order 0..W-1 on every owner: a fixed summation order
      for (int p = 0; p < W; ++p) {
        uint4 raw[U2];
#pragma unroll
        for (int j = 0; j < U2; ++j) {
          const long long u = u0 + j * blockDim.x;
          if (u < hi && p != r) raw[j] = ld_v4_cg(at<TW>(a.data[r], p * cw + (u - r * chunk_u) * V));
        }
#pragma unroll
        for (int j = 0; j < U2; ++j) {
          const long long u = u0 + j * blockDim.x;
          if (u >= hi) continue;
          TA v[V];
          if (p == r) {
            load_in<TI, TA, V>(in + u * V, v);
#pragma unroll
            for (int i = 0; i < V; ++i) v[i] = widen<TA, TW>(narrow<TW, TA>(v[i]));  // same wire rounding as peers'
          } else {
            unpack_vec<TW, TA>(raw[j], v);
          }
#pragma unroll
          for (int i = 0; i < V; ++i) accs[j][i] = p == 0 ? v[i] : combine<OP>(accs[j][i], v[i]);
        }
      }
#pragma unroll
      for (int j = 0; j < U2; ++j) {
      const long long u = u0 + j * blockDim.x;
      if (u >= hi) continue;
      TA* acc = accs[j];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc[i], a.scale)));
      if (sym) {
        // everyone's tensor, chunk r, in the tensor's own type
        TI res[V];
#pragma unroll
        for (int i = 0; i < V; ++i) res[i] = narrow<TI, TA>(acc[i]);
        for (int k = 0; k < W; ++k) {
          const int p = (r + k) % W;
          TI* d = at<TI>(a.dst[p], u * V);
          if constexpr (sizeof(TI) * V == 16) {
            st_v4(d, *reinterpret_cast<const uint4*>(res));
          } else {
#pragma unroll
            for (int i = 0; i < V; ++i) d[i] = res[i];
          }
        }
      } else {
        const uint4 w = pack_vec<TW, TA>(acc);
        for (int k = 1; k < W; ++k) {
          const int p = (r + k) % W;
          st_v4(at<TW>(a.data[p], res_off + u * V), w);
        }
        store_out<TI, TA, V>(out + u * V, acc);
      }
      }
    }
    if (blockIdx.x == 0 && threadIdx.x < tail) {  // every rank reduces the tail itself, in rank order
      const long long e = threadIdx.x;
      TA acc = widen<TA, TW>(*reinterpret_cast<volatile TW*>(at<TW>(a.data[r], tail_off + e)));
      for (int p = 1; p < W; ++p)
        acc = combine<OP>(acc, widen<TA, TW>(*reinterpret_cast<volatile TW*>(at<TW>(a.data[r], tail_off + p * V + e))));
      out[nu * V + e] = narrow<TI, TA>(widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc, a.scale))));
    }
    ok = peer_barrier(a, a.epoch + 2);
  }
  if (ok && !sym) {
    for (int k = 1; k < W; ++k) {
      const int c = (r + k) % W;
      long long lo, hi;
      sub_range(c, &lo, &hi);
      constexpr int U = 4;
      for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
        uint4 w[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const long long u = u0 + j * blockDim.x;
          if (u < hi) w[j] = ld_v4_cg(at<TW>(a.data[r], res_off + u * V));
        }
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const long long u = u0 + j * blockDim.x;
          if (u < hi) {
            TA v[V];
            unpack_vec<TW, TA>(w[j], v);
            store_out<TI, TA, V>(out + u * V, v);
          }
        }
      }
    }
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// reduce-scatter, push: staging [parity 2][W slots][chunk] (wire type)
//   rank r stores chunk c of its input into slot r of rank c, one barrier,
//   then reduces its W local slots into its output chunk.
// ---------------------------------------------------------------------------
template <typename TI, typename TW, int OP>
__global__ void __launch_bounds__(kCommThreads) reduce_scatter_kernel(CommArgs a) {
  using TA = typename Acc<TW>::type;
  constexpr int V = Vec<TW>::n;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long chunk = a.n;
  const long long par = 0;
  const bool vec = chunk % V == 0;
  const TI* in = reinterpret_cast<const TI*>(a.in);
  long long lo, hi;
  block_range(vec ? chunk / V : chunk, &lo, &hi);
  for (int k = 1; k < W; ++k) {  // my own chunk is read from the input in the reduce
    const int c = (r + k) % W;
    if (vec) {
      constexpr int U = 4;
      for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
        uint4 w[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const long long u = u0 + j * blockDim.x;
          if (u < hi) {
            TA v[V];
            load_in<TI, TA, V>(in + c * chunk + u * V, v);
            w[j] = pack_vec<TW, TA>(v);
          }
        }
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const long long u = u0 + j * blockDim.x;
          if (u < hi) st_v4(at<TW>(a.data[c], par + r * chunk + u * V), w[j]);
        }
      }
    } else {
      for (long long e = lo + threadIdx.x; e < hi; e += blockDim.x)
        *at<TW>(a.data[c], par + r * chunk + e) = narrow<TW, TA>(widen<TA, TI>(in[c * chunk + e]));
    }
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  if (ok) {
    TI* out = reinterpret_cast<TI*>(a.out);
    const TI* own = in + r * chunk;
    if (vec) {
      constexpr int U2 = 4;
      for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U2 * blockDim.x) {
        TA accs[U2][V];
        for (int p = 0; p < W; ++p) {  // rank order
          uint4 raw[U2];
#pragma unroll
          for (int j = 0; j < U2; ++j) {
            const long long u = u0 + j * blockDim.x;
            if (u < hi && p != r) raw[j] = ld_v4_cg(at<TW>(a.data[r], par + p * chunk + u * V));
          }
#pragma unroll
          for (int j = 0; j < U2; ++j) {
            const long long u = u0 + j * blockDim.x;
            if (u >= hi) continue;
            TA v[V];
            if (p == r) {
              load_in<TI, TA, V>(own + u * V, v);
#pragma unroll
              for (int i = 0; i < V; ++i) v[i] = widen<TA, TW>(narrow<TW, TA>(v[i]));
            } else {
              unpack_vec<TW, TA>(raw[j], v);
            }
#pragma unroll
            for (int i = 0; i < V; ++i) accs[j][i] = p == 0 ? v[i] : combine<OP>(accs[j][i], v[i]);
          }
        }
#pragma unroll
        for (int j = 0; j < U2; ++j) {
          const long long u = u0 + j * blockDim.x;
          if (u >= hi) continue;
#pragma unroll
          for (int i = 0; i < V; ++i) accs[j][i] = widen<TA, TW>(narrow<TW, TA>(finish<OP>(accs[j][i], a.scale)));
          store_out<TI, TA, V>(out + u * V, accs[j]);
        }
      }
    } else {
      for (long long e = lo + threadIdx.x; e < hi; e += blockDim.x) {
        TA acc = 0;
        for (int p = 0; p < W; ++p) {
          const TA v = p == r ? widen<TA, TW>(narrow<TW, TA>(widen<TA, TI>(own[e])))
                              : widen<TA, TW>(*reinterpret_cast<volatile TW*>(at<TW>(a.data[r], par + p * chunk + e)));
          acc = p == 0 ? v : combine<OP>(acc, v);
        }
        out[e] = narrow<TI, TA>(widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc, a.scale))));
      }
    }
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// reduce-scatter fused with AdamW on the owned shard (FSDP gradients)
//   Phase 1 is the push reduce-scatter above (grad chunk c -> rank c, slot r).
//   Phase 2: each owned element's gradient is summed over the W slots in rank
//   order, scaled (1/W), and used at once for the AdamW update of the fp32
//   master weight and moments; the rounded parameter is written into the
//   shard.  The reduced gradient never goes to memory.
// ---------------------------------------------------------------------------
struct AdamArgs {
  float* master;  // fp32 master shard, or null (parameters are fp32 themselves)
  float* m;
  float* v;
  void* param;    // shard, bf16 or fp32
  float lr, b1, b2, eps, wd, c1, c2;  // c1 = 1 / (1 - b1^t), c2 = 1 / (1 - b2^t)
};

template <bool P_BF16>
MNB_DEVICE void adam_update(const AdamArgs& o, long long e, float g) {
  float w = o.master ? o.master[e]
                     : (P_BF16 ? bf16_to_f32(reinterpret_cast<const __nv_bfloat16*>(o.param)[e])
                               : reinterpret_cast<const float*>(o.param)[e]);
  const float m = o.b1 * o.m[e] + (1.f - o.b1) * g;
  const float v = o.b2 * o.v[e] + (1.f - o.b2) * g * g;
  o.m[e] = m;
  o.v[e] = v;
  w -= o.lr * o.wd * w;
  w -= o.lr * (m * o.c1) / (sqrtf(v * o.c2) + o.eps);
  if (o.master) o.master[e] = w;
  if (P_BF16) reinterpret_cast<__nv_bfloat16*>(o.param)[e] = f32_to_bf16(w);
  else reinterpret_cast<float*>(o.param)[e] = w;
}

// Eight consecutive elements e0..e0+7 (16-byte aligned groups): vector loads
// and stores of the fp32 state and the parameter.
template <bool P_BF16>
MNB_DEVICE void adam_update8(const AdamArgs& o, long long e0, const float* g) {
  float w[8], m[8], v[8];
  auto ld8 = [](const float* p, float* d) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w; d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
  };
  auto st8 = [](float* p, const float* d) {
    *reinterpret_cast<float4*>(p) = make_float4(d[0], d[1], d[2], d[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(d[4], d[5], d[6], d[7]);
  };
  ld8(o.m + e0, m);
  ld8(o.v + e0, v);
  if (o.master) {
    ld8(o.master + e0, w);
  } else if (P_BF16) {
    const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(o.param) + e0);
    const uint32_t rs[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(rs[j]);
      w[2 * j] = f.x;
      w[2 * j + 1] = f.y;
    }
  } else {
    ld8(reinterpret_cast<const float*>(o.param) + e0, w);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m[i] = o.b1 * m[i] + (1.f - o.b1) * g[i];
    v[i] = o.b2 * v[i] + (1.f - o.b2) * g[i] * g[i];
    w[i] -= o.lr * o.wd * w[i];
    w[i] -= o.lr * (m[i] * o.c1) / (sqrtf(v[i] * o.c2) + o.eps);
  }
  st8(o.m + e0, m);
  st8(o.v + e0, v);
  if (o.master) st8(o.master + e0, w);
  if (P_BF16) {
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(o.param) + e0) =
        make_uint4(pack_bf16x2(w[0], w[1]), pack_bf16x2(w[2], w[3]), pack_bf16x2(w[4], w[5]), pack_bf16x2(w[6], w[7]));
  } else {
    st8(reinterpret_cast<float*>(o.param) + e0, w);
  }
}

template <typename TG, bool P_BF16>
__global__ void __launch_bounds__(kCommThreads) rs_adamw_kernel(CommArgs a, AdamArgs o) {
  constexpr int V = Vec<TG>::n;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long chunk = a.n;
  const bool vec = chunk % V == 0;
  const TG* in = reinterpret_cast<const TG*>(a.in);
  long long lo, hi;
  block_range(vec ? chunk / V : chunk, &lo, &hi);
  for (int k = 1; k < W; ++k) {
    const int c = (r + k) % W;
    if (vec) {
      constexpr int U = 4;
      for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
        uint4 w[U];
#pragma unroll
        for (int j = 0; j < U; ++j)
          if (u0 + j * blockDim.x < hi) w[j] = ld_v4(in + c * chunk + (u0 + j * blockDim.x) * V);
#pragma unroll
        for (int j = 0; j < U; ++j)
          if (u0 + j * blockDim.x < hi) st_v4(at<TG>(a.data[c], r * chunk + (u0 + j * blockDim.x) * V), w[j]);
      }
    } else {
      for (long long e = lo + threadIdx.x; e < hi; e += blockDim.x) *at<TG>(a.data[c], r * chunk + e) = in[c * chunk + e];
    }
  }
  const bool ok = peer_barrier(a, a.epoch + 1);
  if (ok) {
    const TG* own = in + r * chunk;
    if (vec) {
      for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
        float g[V];
        for (int p = 0; p < W; ++p) {  // rank order
          float x[V];
          unpack_vec<TG, float>(p == r ? ld_v4(own + u * V) : ld_v4_cg(at<TG>(a.data[r], p * chunk + u * V)), x);
#pragma unroll
          for (int i = 0; i < V; ++i) g[i] = p == 0 ? x[i] : g[i] + x[i];
        }
#pragma unroll
        for (int i = 0; i < V; ++i) g[i] *= a.scale;
        if constexpr (V == 8) {
          adam_update8<P_BF16>(o, u * V, g);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) adam_update<P_BF16>(o, u * V + i, g[i]);
        }
      }
    } else {
      for (long long e = lo + threadIdx.x; e < hi; e += blockDim.x) {
        float g = 0.f;
        for (int p = 0; p < W; ++p) {
          const float x = to_f<TG>(p == r ? own[e] : *reinterpret_cast<volatile TG*>(at<TG>(a.data[r], p * chunk + e)));
          g = p == 0 ? x : g + x;
        }
        adam_update<P_BF16>(o, e, g * a.scale);
      }
    }
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// data movement without reduction, push, byte level (parity-buffered slots):
//   kind 0 all_gather : rank r stores its shard into slot r of every rank
//   kind 1 broadcast  : the root stores the tensor into slot 0 of every rank
//   kind 2 all_to_all : rank r stores its chunk c into slot r of rank c
//   after one barrier every rank copies its slots into its output.
//   n = per-slot bytes (shard / message / chunk)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCommThreads) move_kernel(CommArgs a, int kind) {
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long nb = a.n;
  const int slots = kind == 1 ? 1 : W;
  const long long par = 0;
  const bool v16 = nb % 16 == 0;
  const long long units = v16 ? nb / 16 : nb;
  long long lo, hi;
  block_range(units, &lo, &hi);
  const uint8_t* in = reinterpret_cast<const uint8_t*>(a.in);
  auto push = [&](const uint8_t* src, int peer, int slot) {
    uint8_t* d = reinterpret_cast<uint8_t*>(a.data[peer]) + par + slot * nb;
    if (!v16) {
      for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) d[u] = src[u];
      return;
    }
    constexpr int U = 4;
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
      uint4 w[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * blockDim.x < hi) w[j] = ld_v4(src + 16 * (u0 + j * blockDim.x));
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * blockDim.x < hi) st_v4(d + 16 * (u0 + j * blockDim.x), w[j]);
    }
  };
  if (kind == 0) {
    for (int k = 0; k < W; ++k) push(in, (r + k) % W, r);
  } else if (kind == 1) {
    if (r == a.root)
      for (int k = 1; k < W; ++k) push(in, (r + k) % W, 0);
  } else {
    for (int k = 0; k < W; ++k) {
      const int c = (r + k) % W;
      push(in + c * nb, c, r);
    }
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  if (ok) {
    uint8_t* out = reinterpret_cast<uint8_t*>(a.out);
    const uint8_t* mine = reinterpret_cast<const uint8_t*>(a.data[r]) + par;
    for (int s = 0; s < slots; ++s) {
      const uint8_t* src;
      uint8_t* dst;
      if (kind == 1) {
        if (r == a.root) {
          if (a.out == a.in) break;
          src = in;
        } else {
          src = mine;
        }
        dst = out;
      } else {
        src = mine + s * nb;
        dst = out + s * nb;
      }
      if (!v16) {
        for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x)
          dst[u] = *reinterpret_cast<const volatile uint8_t*>(src + u);
        continue;
      }
      constexpr int U = 4;
      for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
        uint4 w[U];
#pragma unroll
        for (int j = 0; j < U; ++j)
          if (u0 + j * blockDim.x < hi) w[j] = ld_v4_cg(src + 16 * (u0 + j * blockDim.x));
#pragma unroll
        for (int j = 0; j < U; ++j)
          if (u0 + j * blockDim.x < hi) st_v4(dst + 16 * (u0 + j * blockDim.x), w[j]);
      }
    }
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// broadcast as scatter + all-gather (W >= 4): the root's NVLink egress would
// otherwise carry (W-1) copies of the message.
//   phase A  the root stores chunk c of the message into rank c's staging
//   phase B  rank c stores chunk c into every other non-root rank's staging
//            (the root sends its own chunk from its input)
//   phase C  non-root ranks copy the staging out.
// Every rank's egress is about one message.  Each block moves the same
// sub-range of every chunk in every phase, so the per-block barriers order
// exactly the data that block depends on.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCommThreads) bcast_scatter_gather_kernel(CommArgs a) {
  ring_begin(a);
  const int W = a.world, r = a.rank, root = a.root;
  const long long nb = a.n;
  const bool v16 = nb % 16 == 0;
  const long long unit = v16 ? 16 : 1;
  const long long units = nb / unit;
  const long long cu = (units + W - 1) / W;  // units per chunk
  const long long sub = (cu + gridDim.x - 1) / gridDim.x;
  const uint8_t* in = reinterpret_cast<const uint8_t*>(a.in);
  auto range = [&](int c, long long* lo, long long* hi) {  // this block's units of chunk c
    const long long c0 = min(units, c * cu), c1 = min(units, c0 + cu);
    *lo = min(c1, c0 + sub * blockIdx.x);
    *hi = min(c1, *lo + sub);
  };
  auto copy = [&](const uint8_t* src, uint8_t* dst, long long lo, long long hi, bool volatile_src) {
    if (!v16) {
      for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x)
        dst[u] = volatile_src ? *reinterpret_cast<const volatile uint8_t*>(src + u) : src[u];
      return;
    }
    constexpr int U = 4;
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
      uint4 w[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * blockDim.x < hi)
          w[j] = volatile_src ? ld_v4_cg(src + 16 * (u0 + j * blockDim.x)) : ld_v4(src + 16 * (u0 + j * blockDim.x));
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * blockDim.x < hi) st_v4(dst + 16 * (u0 + j * blockDim.x), w[j]);
    }
  };
  long long lo, hi;
  if (r == root) {
    for (int k = 1; k < W; ++k) {
      const int c = (r + k) % W;
      range(c, &lo, &hi);
      copy(in, reinterpret_cast<uint8_t*>(a.data[c]), lo, hi, false);
    }
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  if (ok) {
    range(r, &lo, &hi);
    const uint8_t* src = r == root ? in : reinterpret_cast<const uint8_t*>(a.data[r]);
    for (int k = 1; k < W; ++k) {
      const int p = (r + k) % W;
      if (p != root) copy(src, reinterpret_cast<uint8_t*>(a.data[p]), lo, hi, r != root);
    }
    ok = peer_barrier(a, a.epoch + 2);
  }
  if (ok) {
    uint8_t* out = reinterpret_cast<uint8_t*>(a.out);
    for (int c = 0; c < W; ++c) {
      range(c, &lo, &hi);
      if (r != root) copy(reinterpret_cast<const uint8_t*>(a.data[r]), out, lo, hi, true);
      else if (a.out != a.in) copy(in, out, lo, hi, false);
    }
  }
  ring_end(a, ok);
}

// ===========================================================================
// NVLS collectives: multimem loads and stores through an NVSwitch multicast
// address (nvls.h).  `uc` / `mc` are the unicast and multicast addresses of
// the same bytes of this call's region: a symmetric NVLS tensor (in place) or
// the NVLS staging buffer (one parity half per call, like the peer staging).
//
// Work split: the message is W slices; block b of every rank owns sub-range
// b of every slice, so a block-level barrier (block b of every rank) orders
// exactly the bytes that block touches.  Rank r reduces slice r:
//   multimem.ld_reduce  the NVSwitch reads slice r from every rank's memory
//                       and returns the sum (bf16 / f16 accumulated in fp32);
//   multimem.st         writes the result into every rank's memory at once.
// Each element is reduced once, by one rank, so every rank holds identical
// bits.  Per GPU that moves about (1 + 1/W) x the message over NVLink in each
// direction, against 2 (W-1)/W for the peer two-shot kernel.
// Accesses through the unicast and the multicast address of the same memory
// are ordered with fence.proxy.alias around every barrier.
// ===========================================================================
MNB_DEVICE void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

MNB_DEVICE bool nvls_barrier(const CommArgs& a, uint32_t value) {
  fence_proxy_alias();
  const bool ok = peer_barrier(a, value);
  fence_proxy_alias();
  return ok;
}

template <typename T> struct Multimem;
template <> struct Multimem<float> {
  static MNB_DEVICE uint4 ld_reduce(const void* p) {
    float4 f;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w)
                 : "l"(p)
                 : "memory");
    return make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z), __float_as_uint(f.w));
  }
  static MNB_DEVICE void unpack(uint4 v, float* f) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y); f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  }
  static MNB_DEVICE uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};
template <> struct Multimem<__nv_bfloat16> {
  static MNB_DEVICE uint4 ld_reduce(const void* p) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
  }
  static MNB_DEVICE void unpack(uint4 v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = unpack_bf16x2(w[j]);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
  static MNB_DEVICE uint4 pack(const float* f) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
  }
};
template <> struct Multimem<__half> {
  static MNB_DEVICE uint4 ld_reduce(const void* p) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
  }
  static MNB_DEVICE void unpack(uint4 v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
  static MNB_DEVICE uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 h = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

// 16 bytes into every rank's memory (raw bits: a store does no arithmetic).
MNB_DEVICE void multimem_st16(void* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(__uint_as_float(v.x)),
               "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)), "f"(__uint_as_float(v.w))
               : "memory");
}

// Sub-range of slice c owned by this block, in 16-byte units.
struct SliceSplit {
  long long units, per_slice, per_block;
  MNB_DEVICE void range(int c, long long* lo, long long* hi) const {
    const long long c0 = min(units, c * per_slice), c1 = min(units, c0 + per_slice);
    *lo = min(c1, c0 + per_block * blockIdx.x);
    *hi = min(c1, *lo + per_block);
  }
};
MNB_DEVICE SliceSplit slice_split(long long units, int slices) {
  SliceSplit s;
  s.units = units;
  s.per_slice = (units + slices - 1) / slices;
  s.per_block = (s.per_slice + gridDim.x - 1) / gridDim.x;
  return s;
}

// Copy 16-byte units [lo, hi) of an n-element array; the last unit may be
// partial: into the staging region it is zero-padded, out of it only the
// n elements are written.
template <typename T>
MNB_DEVICE void copy_units(const T* src, T* dst, long long lo, long long hi, long long n, bool pad) {
  constexpr int V = 16 / sizeof(T);
  constexpr int U = 4;
  for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
    uint4 w[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const long long u = u0 + j * blockDim.x;
      if (u < hi && (u + 1) * V <= n) w[j] = ld_v4_cg(src + u * V);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const long long u = u0 + j * blockDim.x;
      if (u >= hi) continue;
      if ((u + 1) * V <= n) {
        st_v4(dst + u * V, w[j]);
      } else {
        for (int i = 0; i < V; ++i) {
          const long long e = u * V + i;
          if (e < n) dst[e] = src[e];
          else if (pad) dst[e] = T(0.0f);
        }
      }
    }
  }
}

// Copy 16-byte units [lo, hi) (byte moves; sizes are 16-byte multiples).
MNB_DEVICE void copy16(const void* src, void* dst, long long lo, long long hi) {
  const uint8_t* s8 = reinterpret_cast<const uint8_t*>(src);
  uint8_t* d8 = reinterpret_cast<uint8_t*>(dst);
  constexpr int U = 4;
  for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * blockDim.x) {
    uint4 w[U];
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (u0 + j * blockDim.x < hi) w[j] = ld_v4_cg(s8 + 16 * (u0 + j * blockDim.x));
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (u0 + j * blockDim.x < hi) st_v4(d8 + 16 * (u0 + j * blockDim.x), w[j]);
  }
}

// all-reduce (sum).  staged: copy the input into the region first and the
// result out of it last; otherwise the tensor is the region (in place).
template <typename T, int THREADS, int MINB>
__global__ void __launch_bounds__(THREADS, MINB) nvls_all_reduce_kernel(CommArgs a, char* uc, char* mc, int staged) {
  constexpr int V = 16 / sizeof(T);
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long n = a.n;
  const SliceSplit sp = slice_split((n + V - 1) / V, W);
  long long lo, hi;
  if (staged) {
    for (int c = 0; c < W; ++c) {
      sp.range(c, &lo, &hi);
      copy_units<T>(reinterpret_cast<const T*>(a.in), reinterpret_cast<T*>(uc), lo, hi, n, true);
    }
  }
  bool ok = nvls_barrier(a, a.epoch + 1);
  if (ok) {
    sp.range(r, &lo, &hi);
    constexpr int U = 4;  // independent multimem loads in flight per thread
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * THREADS) {
      uint4 v[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * THREADS < hi) v[j] = Multimem<T>::ld_reduce(mc + 16 * (u0 + j * THREADS));
#pragma unroll
      for (int j = 0; j < U; ++j) {
        if (u0 + j * THREADS >= hi) continue;
        if (a.scale != 1.0f) {
          float f[V];
          Multimem<T>::unpack(v[j], f);
#pragma unroll
          for (int i = 0; i < V; ++i) f[i] *= a.scale;
          v[j] = Multimem<T>::pack(f);
        }
        multimem_st16(mc + 16 * (u0 + j * THREADS), v[j]);
      }
    }
    ok = nvls_barrier(a, a.epoch + 2);
  }
  if (ok && staged) {
    for (int c = 0; c < W; ++c) {
      sp.range(c, &lo, &hi);
      copy_units<T>(reinterpret_cast<const T*>(uc), reinterpret_cast<T*>(a.out), lo, hi, n, false);
    }
  }
  ring_end(a, ok);
}

// reduce-scatter (sum): out[chunk] = scale * sum over ranks of chunk r of the
// input.  a.n = chunk elements (16-byte multiple).  The trailing barrier keeps
// a fast rank from refilling its input while a peer's reduction still reads it.
template <typename T>
__global__ void __launch_bounds__(kCommThreads) nvls_reduce_scatter_kernel(CommArgs a, char* uc, char* mc, int staged) {
  constexpr int V = 16 / sizeof(T);
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long chunk_u = a.n / V;
  const SliceSplit sp = slice_split(chunk_u * W, W);
  long long lo, hi;
  if (staged) {
    for (int c = 0; c < W; ++c) {
      sp.range(c, &lo, &hi);
      copy_units<T>(reinterpret_cast<const T*>(a.in), reinterpret_cast<T*>(uc), lo, hi, a.n * W, true);
    }
  }
  bool ok = nvls_barrier(a, a.epoch + 1);
  if (ok) {
    sp.range(r, &lo, &hi);
    T* out = reinterpret_cast<T*>(a.out);
    constexpr int U = 4;
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * kCommThreads) {
      uint4 v[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * kCommThreads < hi) v[j] = Multimem<T>::ld_reduce(mc + 16 * (u0 + j * kCommThreads));
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const long long u = u0 + j * kCommThreads;
        if (u >= hi) continue;
        if (a.scale != 1.0f) {
          float f[V];
          Multimem<T>::unpack(v[j], f);
#pragma unroll
          for (int i = 0; i < V; ++i) f[i] *= a.scale;
          v[j] = Multimem<T>::pack(f);
        }
        st_v4(out + (u - r * chunk_u) * V, v[j]);
      }
    }
    ok = nvls_barrier(a, a.epoch + 2);
  }
  ring_end(a, ok);
}

// reduce-scatter fused with AdamW on the owned shard: the switch returns the
// summed gradient slice and it feeds the update directly (see rs_adamw_kernel).
template <typename TG, bool P_BF16>
__global__ void __launch_bounds__(kCommThreads) nvls_rs_adamw_kernel(CommArgs a, AdamArgs o, char* uc, char* mc,
                                                                    int staged) {
  constexpr int V = 16 / sizeof(TG);
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long chunk_u = a.n / V;
  const SliceSplit sp = slice_split(chunk_u * W, W);
  long long lo, hi;
  if (staged) {
    for (int c = 0; c < W; ++c) {
      sp.range(c, &lo, &hi);
      copy_units<TG>(reinterpret_cast<const TG*>(a.in), reinterpret_cast<TG*>(uc), lo, hi, a.n * W, true);
    }
  }
  bool ok = nvls_barrier(a, a.epoch + 1);
  if (ok) {
    sp.range(r, &lo, &hi);
    for (long long u = lo + threadIdx.x; u < hi; u += kCommThreads) {
      float g[8];
      Multimem<TG>::unpack(Multimem<TG>::ld_reduce(mc + 16 * u), g);
#pragma unroll
      for (int i = 0; i < V; ++i) g[i] *= a.scale;
      const long long e0 = (u - r * chunk_u) * V;
      if constexpr (V == 8) {
        adam_update8<P_BF16>(o, e0, g);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) adam_update<P_BF16>(o, e0 + i, g[i]);
      }
    }
    ok = nvls_barrier(a, a.epoch + 2);
  }
  ring_end(a, ok);
}

// all-gather (kind 0: every rank stores its shard into slot r of every rank)
// and broadcast (kind 1: the root stores the message into every rank), by
// multimem stores; a.n = bytes per slot (16-byte multiple).  A first barrier
// makes sure every rank is inside this collective before any store reaches
// its memory (no multimem access ever targets a rank that has not launched
// the same kernel); after the second one each rank copies the region out.
__global__ void __launch_bounds__(kCommThreads) nvls_move_kernel(CommArgs a, char* uc, char* mc, int kind) {
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long units = a.n / 16;
  const int slots = kind == 0 ? W : 1;
  const SliceSplit sp = slice_split(units, 1);
  long long lo, hi;
  sp.range(0, &lo, &hi);
  const uint8_t* in = reinterpret_cast<const uint8_t*>(a.in);
  bool ok = nvls_barrier(a, a.epoch + 1);
  if (ok && (kind == 0 || r == a.root)) {
    char* dst = mc + (kind == 0 ? r * a.n : 0);
    constexpr int U = 4;
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * kCommThreads) {
      uint4 w[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * kCommThreads < hi) w[j] = ld_v4(in + 16 * (u0 + j * kCommThreads));
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * kCommThreads < hi) multimem_st16(dst + 16 * (u0 + j * kCommThreads), w[j]);
    }
  }
  if (ok) ok = nvls_barrier(a, a.epoch + 2);
  if (ok) {
    uint8_t* out = reinterpret_cast<uint8_t*>(a.out);
    for (int s = 0; s < slots; ++s) {
      if (kind == 1 && r == a.root) {
        if (a.out != a.in) copy16(in, out, lo, hi);
        break;
      }
      copy16(uc + s * a.n, out + s * a.n, lo, hi);
    }
  }
  ring_end(a, ok);
}

// ===========================================================================
// DDP with the optimizer inside the gradient reduction (one kernel per
// bucket; ZeRO-1 layout): rank r owns elements [r*slice, (r+1)*slice) of the
// bucket -- it reduces their gradients, applies AdamW to them with fp32
// master weights and moments held for that slice only, and writes the new
// parameters (the bucket's type) into every rank's parameter bucket.  The
// traffic is a reduce-scatter of gradients plus an all-gather of parameters,
// the same bytes as the all-reduce it replaces, and the optimizer work and
// state shrink W-fold.  a.n = slice (elements, a multiple of 16 / sizeof(T)).
// ===========================================================================
template <typename T> struct Pack;
template <> struct Pack<__nv_bfloat16> {
  static constexpr int V = 8;
  static MNB_DEVICE void unpack(uint4 v, float* f) { Multimem<__nv_bfloat16>::unpack(v, f); }
  static MNB_DEVICE uint4 pack(const float* f) { return Multimem<__nv_bfloat16>::pack(f); }
};
template <> struct Pack<float> {
  static constexpr int V = 4;
  static MNB_DEVICE void unpack(uint4 v, float* f) { Multimem<float>::unpack(v, f); }
  static MNB_DEVICE uint4 pack(const float* f) { return Multimem<float>::pack(f); }
};

// AdamW on V consecutive slice elements starting at e0 (state arrays index
// the slice); g holds the reduced, scaled gradients; w receives the new weights.
template <int V>
MNB_DEVICE void adamw_slice(const AdamArgs& o, long long e0, const float* g, float* w) {
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const long long e = e0 + i;
    const float m = o.b1 * o.m[e] + (1.f - o.b1) * g[i];
    const float v = o.b2 * o.v[e] + (1.f - o.b2) * g[i] * g[i];
    o.m[e] = m;
    o.v[e] = v;
    float x = o.master[e];
    x -= o.lr * o.wd * x;
    x -= o.lr * (m * o.c1) / (sqrtf(v * o.c2) + o.eps);
    o.master[e] = x;
    w[i] = x;
  }
}

// Peer-memory version: phase 1 pushes gradient chunk c into rank c's staging
// slot r; phase 2 sums the owned chunk in rank order (identical bits on every
// rank), updates it and stores the parameters into every rank's bucket
// (a.dst[p] = rank p's parameter bucket).
template <typename T, int THREADS, int MINB>
__global__ void __launch_bounds__(THREADS, MINB) ar_adamw_push_kernel(CommArgs a, AdamArgs o) {
  constexpr int V = Pack<T>::V;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long slice_u = a.n / V;
  const SliceSplit sp = slice_split(slice_u * W, W);
  const T* in = reinterpret_cast<const T*>(a.in);
  long long lo, hi;
  for (int k = 1; k < W; ++k) {  // my copy of chunk c -> slot r of rank c
    const int c = (r + k) % W;
    sp.range(c, &lo, &hi);
    const uint4* src = reinterpret_cast<const uint4*>(in) + c * slice_u;
    uint4* dst = reinterpret_cast<uint4*>(a.data[c]) + r * slice_u;
    constexpr int U = 4;
    for (long long u0 = lo - c * slice_u + threadIdx.x; u0 < hi - c * slice_u; u0 += U * THREADS) {
      uint4 w[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * THREADS < hi - c * slice_u) w[j] = ld_v4(src + u0 + j * THREADS);
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * THREADS < hi - c * slice_u) st_v4(dst + u0 + j * THREADS, w[j]);
    }
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  if (ok) {
    sp.range(r, &lo, &hi);
    constexpr int U = 2;  // units per thread with all their slot loads in flight
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * THREADS) {
      float g[U][V];
      for (int q = 0; q < W; ++q) {  // rank order
        uint4 raw[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const long long u = u0 + j * THREADS;
          if (u < hi)
            raw[j] = q == r ? ld_v4(in + u * V)
                            : ld_v4_cg(reinterpret_cast<const T*>(a.data[r]) + static_cast<long long>(q) * a.n +
                                       (u - r * slice_u) * V);
        }
#pragma unroll
        for (int j = 0; j < U; ++j) {
          float x[V];
          Pack<T>::unpack(raw[j], x);
#pragma unroll
          for (int i = 0; i < V; ++i) g[j][i] = q == 0 ? x[i] : g[j][i] + x[i];
        }
      }
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const long long u = u0 + j * THREADS;
        if (u >= hi) continue;
#pragma unroll
        for (int i = 0; i < V; ++i) g[j][i] *= a.scale;
        float w[V];
        adamw_slice<V>(o, (u - r * slice_u) * V, g[j], w);
        const uint4 pw = Pack<T>::pack(w);
        for (int k = 0; k < W; ++k) st_v4(reinterpret_cast<T*>(a.dst[(r + k) % W]) + u * V, pw);
      }
    }
    ok = peer_barrier(a, a.epoch + 2);
  }
  ring_end(a, ok);
}

// NVLS version: the switch returns the summed gradient slice, the new
// parameters go to every rank with one multimem store.  U switch loads per
// thread are in flight before the first update (each waits a round trip).
template <typename T, int THREADS, int MINB>
__global__ void __launch_bounds__(THREADS, MINB) nvls_ar_adamw_kernel(CommArgs a, AdamArgs o, char* g_mc,
                                                                       char* p_mc) {
  constexpr int V = Pack<T>::V;
  constexpr int U = 4;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long slice_u = a.n / V;
  const SliceSplit sp = slice_split(slice_u * W, W);
  bool ok = nvls_barrier(a, a.epoch + 1);
  if (ok) {
    long long lo, hi;
    sp.range(r, &lo, &hi);
    for (long long u0 = lo + threadIdx.x; u0 < hi; u0 += U * THREADS) {
      uint4 raw[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * THREADS < hi) raw[j] = Multimem<T>::ld_reduce(g_mc + 16 * (u0 + j * THREADS));
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const long long u = u0 + j * THREADS;
        if (u >= hi) continue;
        float g[V], w[V];
        Multimem<T>::unpack(raw[j], g);
#pragma unroll
        for (int i = 0; i < V; ++i) g[i] *= a.scale;
        adamw_slice<V>(o, (u - r * slice_u) * V, g, w);
        multimem_st16(p_mc + 16 * u, Pack<T>::pack(w));
      }
    }
    ok = nvls_barrier(a, a.epoch + 2);
  }
  ring_end(a, ok);
}

__global__ void barrier_kernel(CommArgs a) {
  ring_begin(a);
  const bool ok = peer_barrier(a, a.epoch + 1);
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// stepped executor (ring / tree / halving / naive schedules)
//   steps: int64 [S][5] = {peer, src_off, dst_off, count, mode}, mode 0 idle,
//   1 dst += wire(peer[src]), 2 dst = peer[src].  Working buffer (type TK)
//   is data[rank]; with `round_bf16` every value read from a peer is rounded
//   to bf16 first, reproducing a narrow wire hop by hop.
// ---------------------------------------------------------------------------
MNB_DEVICE bool grid_peer_barrier(const CommArgs& a, uint32_t value, cg::grid_group& grid) {
  grid.sync();
  __shared__ int flag;
  if (blockIdx.x == 0) {
    const bool ok = peer_barrier(a, value);
    if (threadIdx.x == 0) flag = ok;
  }
  grid.sync();
  return a.status[0] == 0;
}

template <typename TI, typename TK, int OP>
__global__ void __launch_bounds__(kCommThreads) stepped_kernel(CommArgs a, const long long* steps, int n_steps,
                                                               int round_bf16) {
  using TA = typename Acc<TK>::type;
  cg::grid_group grid = cg::this_grid();
  ring_begin(a);
  TK* work = reinterpret_cast<TK*>(a.data[a.rank]);
  const long long n = a.n;
  const long long gt = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long gs = static_cast<long long>(gridDim.x) * blockDim.x;
  const TI* in = reinterpret_cast<const TI*>(a.in);
  for (long long e = gt; e < n; e += gs) work[e] = narrow<TK, TA>(widen<TA, TI>(in[e]));
  bool ok = grid_peer_barrier(a, a.epoch + 1, grid);
  for (int s = 0; s < n_steps && ok; ++s) {
    const long long* st = steps + 5 * s;
    const int mode = static_cast<int>(st[4]);
    if (mode != 0) {
      const TK* src = reinterpret_cast<const TK*>(a.data[st[0]]) + st[1];
      TK* dst = work + st[2];
      for (long long e = gt; e < st[3]; e += gs) {
        TA x = widen<TA, TK>(src[e]);
        if (round_bf16) x = static_cast<TA>(__bfloat162float(__float2bfloat16_rn(static_cast<float>(x))));
        dst[e] = mode == 1 ? narrow<TK, TA>(combine<OP>(widen<TA, TK>(dst[e]), x)) : narrow<TK, TA>(x);
      }
    }
    ok = grid_peer_barrier(a, a.epoch + 2 + s, grid);
  }
  if (ok) {
    TI* out = reinterpret_cast<TI*>(a.out);
    for (long long e = gt; e < n; e += gs) out[e] = narrow<TI, TA>(finish<OP>(widen<TA, TK>(work[e]), a.scale));
  }
  if (ok) ok = grid_peer_barrier(a, a.epoch + 2 + n_steps, grid);  // peers done reading my work buffer
  grid.sync();
  ring_end(a, ok);
}

// ===========================================================================
// host runtime
// ===========================================================================
namespace {

void ck(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

std::string ipc_bytes(void* p) {
  cudaIpcMemHandle_t h;
  ck(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void* ipc_open(const std::string& bytes) {
  TORCH_CHECK(bytes.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, bytes.data(), sizeof(h));
  void* p = nullptr;
  ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return p;
}

}  // namespace

// tcgen05 GEMM fused with a reduce-scatter (fuse 1) or an all-gather (fuse 2); gemm.cu.
void gemm_fused(int fuse, torch::Tensor a, torch::Tensor b, torch::Tensor out, bool b_mn,
                c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux,
                c10::optional<torch::Tensor> resid, int64_t epi, torch::Tensor status, const PeerCtx& ctx,
                uint32_t* ag_base, c10::optional<torch::Tensor> stamps);

// FSDP weight all-gather fused with the GEMM that consumes it; gemm.cu.
void gemm_agw(torch::Tensor x, torch::Tensor flat, int64_t w_off, int64_t N, c10::optional<torch::Tensor> bias,
              torch::Tensor out, const std::vector<const void*>& shards, int64_t shard, torch::Tensor counters,
              torch::Tensor status, const PeerCtx& ctx, uint32_t* ag_base);

struct Segment {
  void* local = nullptr;
  int64_t bytes = 0;
  std::vector<void*> peers;  // peers[r]; own rank = local
  bool opened = false;
};

class DeviceCommImpl {
 public:
  DeviceCommImpl(int rank, int world, int device, int64_t staging_bytes)
      : rank_(rank), world_(world), device_(device) {
    TORCH_CHECK(world >= 1 && world <= kMaxRanks, "device communicator supports 1..16 ranks");
    c10::cuda::CUDAGuard g(device);
    ck(cudaMalloc(&sig_local_, kSigSlots * sizeof(uint32_t)), "cudaMalloc(signals)");
    ck(cudaMemset(sig_local_, 0, kSigSlots * sizeof(uint32_t)), "cudaMemset(signals)");
    void* sh = nullptr;
    ck(cudaHostAlloc(&sh, 16 * sizeof(int), cudaHostAllocMapped), "status");
    status_h_ = static_cast<volatile int*>(sh);
    std::memset(const_cast<int*>(status_h_), 0, 16 * sizeof(int));
    void* sd = nullptr;
    ck(cudaHostGetDevicePointer(&sd, const_cast<int*>(status_h_), 0), "status ptr");
    status_d_ = static_cast<volatile int*>(sd);
    ck(cudaHostAlloc(reinterpret_cast<void**>(&ring_h_), kRingCap * sizeof(DevEvent), cudaHostAllocMapped), "ring");
    std::memset(ring_h_, 0, kRingCap * sizeof(DevEvent));
    ck(cudaHostGetDevicePointer(reinterpret_cast<void**>(&ring_d_), ring_h_, 0), "ring ptr");
    staging_ = add_segment(staging_bytes);
    sig_peers_.assign(world, nullptr);
    sig_peers_[rank] = static_cast<uint32_t*>(sig_local_);
    ck(cudaDeviceSynchronize(), "init sync");
  }

  ~DeviceCommImpl() { close(); }

  void close() {
    if (closed_) return;
    closed_ = true;
    c10::cuda::CUDAGuard g(device_);
    cudaDeviceSynchronize();
    for (auto& o : nvls_) o->release();  // the Python layer synchronised every rank first
    nvls_.clear();
    nvls_staging_ = -1;
    for (auto& s : segs_) {
      for (int r = 0; r < world_; ++r)
        if (r != rank_ && s.opened && s.peers[r]) cudaIpcCloseMemHandle(s.peers[r]);
      if (s.local) cudaFree(s.local);
    }
    for (int r = 0; r < world_; ++r)
      if (r != rank_ && sig_opened_ && sig_peers_[r]) cudaIpcCloseMemHandle(sig_peers_[r]);
    if (sig_local_) cudaFree(sig_local_);
    if (status_h_) cudaFreeHost(const_cast<int*>(status_h_));
    if (ring_h_) cudaFreeHost(ring_h_);
    segs_.clear();
  }

  // ---- handle exchange ---------------------------------------------------
  int add_segment(int64_t bytes) {
    c10::cuda::CUDAGuard g(device_);
    Segment s;
    s.bytes = std::max<int64_t>(bytes, 256);
    ck(cudaMalloc(&s.local, s.bytes), "cudaMalloc(segment)");
    ck(cudaMemset(s.local, 0, s.bytes), "cudaMemset(segment)");
    s.peers.assign(world_, nullptr);
    s.peers[rank_] = s.local;
    if (world_ == 1) s.opened = true;
    segs_.push_back(s);
    return static_cast<int>(segs_.size()) - 1;
  }
  py::bytes segment_handle(int id) { return py::bytes(ipc_bytes(segs_.at(id).local)); }
  py::bytes signal_handle() { return py::bytes(ipc_bytes(sig_local_)); }
  void open_segment(int id, std::vector<std::string> handles) {
    c10::cuda::CUDAGuard g(device_);
    Segment& s = segs_.at(id);
    TORCH_CHECK(static_cast<int>(handles.size()) == world_, "need one handle per rank");
    for (int r = 0; r < world_; ++r)
      if (r != rank_) s.peers[r] = ipc_open(handles[r]);
    s.opened = true;
  }
  void open_signals(std::vector<std::string> handles) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(static_cast<int>(handles.size()) == world_, "need one handle per rank");
    for (int r = 0; r < world_; ++r)
      if (r != rank_) sig_peers_[r] = static_cast<uint32_t*>(ipc_open(handles[r]));
    sig_opened_ = true;
  }
  uintptr_t segment_ptr(int id) { return reinterpret_cast<uintptr_t>(segs_.at(id).local); }
  int64_t segment_bytes(int id) { return segs_.at(id).bytes; }
  int staging_segment() const { return staging_; }
  void set_staging(int id) {
    TORCH_CHECK(id >= 0 && id < static_cast<int>(segs_.size()) && segs_[id].opened, "bad staging segment");
    staging_ = id;
  }
  // View of a segment as a tensor; the memory is owned by this communicator.
  torch::Tensor segment_tensor(int id, int64_t numel, at::ScalarType dtype) {
    const Segment& s = segs_.at(id);
    auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device_);
    TORCH_CHECK(numel * static_cast<int64_t>(c10::elementSize(dtype)) <= s.bytes, "segment too small");
    return torch::from_blob(s.local, {numel}, [](void*) {}, opts);
  }

  // Which segment (and offset) holds [p, p+bytes)?  -1 if none.
  std::pair<int, int64_t> locate(const void* p, int64_t bytes) const {
    const auto a = reinterpret_cast<uintptr_t>(p);
    for (size_t i = 0; i < segs_.size(); ++i) {
      const auto b = reinterpret_cast<uintptr_t>(segs_[i].local);
      if (a >= b && a + bytes <= b + segs_[i].bytes) return {static_cast<int>(i), static_cast<int64_t>(a - b)};
    }
    return {-1, 0};
  }
  bool is_symmetric(torch::Tensor t) {
    return locate(t.data_ptr(), t.numel() * t.element_size()).first >= 0;
  }

  // ---- status / event ring -------------------------------------------------
  std::vector<int> status() const { return {status_h_[0], status_h_[1], status_h_[2], status_h_[3]}; }
  void clear_status() { for (int i = 0; i < 4; ++i) const_cast<int*>(status_h_)[i] = 0; }
  void set_timeout(double seconds) { timeout_ns_ = static_cast<unsigned long long>(seconds * 1e9); }
  uint32_t seq() const { return seq_; }
  py::list events(int64_t last) const {
    py::list out;
    const uint32_t first = seq_ > static_cast<uint32_t>(std::min<int64_t>(last, kRingCap)) ? seq_ - static_cast<uint32_t>(std::min<int64_t>(last, kRingCap)) : 0;
    for (uint32_t s = first; s < seq_; ++s) {
      const DevEvent& e = ring_h_[s % kRingCap];
      if (e.seq != s || e.t_start == 0) continue;
      py::dict d;
      d["seq"] = e.seq;
      d["opcode"] = e.op;
      d["nbytes"] = e.nbytes;
      d["start_ns"] = e.t_start;
      d["end_ns"] = e.t_end;
      d["status"] = e.status;
      out.append(d);
    }
    return out;
  }

  // ---- launch helpers ----------------------------------------------------------
  CommArgs base_args(int seg, int64_t offset, const void* in, void* out, long long n, int opname, long long nbytes,
                     int barriers) {
    CommArgs a{};
    const Segment& s = segs_.at(seg);
    TORCH_CHECK(s.opened, "symmetric segment not mapped on every rank yet");
    TORCH_CHECK(sig_opened_ || world_ == 1, "signal pads not mapped");
    // Calls alternate between the two halves of the staging buffer, so a peer
    // that has already moved on to the next call never writes into memory
    // this rank is still reading (call k+2 cannot start before every rank
    // has entered call k+1).
    const int64_t half = seg == staging_ ? (s.bytes / 2) / 256 * 256 : 0;
    const int64_t par_off = seg == staging_ ? static_cast<int64_t>(seq_ & 1) * half : 0;
    for (int r = 0; r < world_; ++r) {
      a.data[r] = static_cast<uint8_t*>(s.peers[r]) + offset + par_off;
      a.sig[r] = sig_peers_[r];
    }
    a.in = in;
    a.out = out;
    a.n = n;
    a.rank = rank_;
    a.world = world_;
    a.epoch = epoch_;
    epoch_ += static_cast<uint32_t>(barriers + 1);
    a.scale = 1.0f;
    a.status = status_d_;
    a.timeout_ns = timeout_ns_;
    a.ring = ring_d_;
    a.seq = seq_++;
    a.opname = opname;
    a.nbytes = nbytes;
    return a;
  }

  int blocks_for(int64_t bytes, int max_blocks, int64_t per_cta = 64 << 10) const {
    int64_t b = (bytes + per_cta - 1) / per_cta;  // ~64 KiB per 512-thread CTA per call
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(b, std::min(max_blocks, kMaxCommBlocks))));
  }

  // Staging bytes a call needs (wire elements of `wsz` bytes); mirrors the
  // layouts documented on each kernel.  kind: 0 one-shot AR, 1 two-shot AR,
  // 2 reduce-scatter (n = input elements), 3 all_gather / all_to_all
  // (n = bytes per rank), 4 broadcast (n = bytes).
  int64_t staging_need(int kind, int64_t n, int64_t wsz) const {
    const int64_t W = world_;
    const int64_t V = 16 / std::max<int64_t>(1, wsz);
    // Each call uses one half of the staging buffer: the need is doubled.
    switch (kind) {
      case 0: return 2 * W * ((n + V - 1) / V * V) * wsz;
      case 1: {
        const int64_t chunk_u = ((n / V) + W - 1) / W;
        return 2 * (2 * W * chunk_u * V + W * V) * wsz;
      }
      case 2: return 2 * n * wsz;
      case 3: return 2 * W * n;
      case 5: return 2 * n * wsz;  // stepped schedules: one working copy
      default: return 2 * n;
    }
  }

  static PeerCtx peer_ctx(const CommArgs& a) {
    PeerCtx c{};
    for (int r = 0; r < a.world; ++r) {
      c.data[r] = a.data[r];
      c.sig[r] = a.sig[r];
    }
    c.rank = a.rank;
    c.world = a.world;
    c.epoch = a.epoch;
    c.seq = a.seq;
    c.status = a.status;
    c.timeout_ns = a.timeout_ns;
    return c;
  }

  // out[M/W, N] = (sum over ranks of x_r @ w_r^T)[this rank's rows] + bias + resid,
  // as one kernel: tiles are pushed to their owners as they finish.
  void gemm_rs(torch::Tensor x, torch::Tensor w, torch::Tensor out, bool w_mn, c10::optional<torch::Tensor> bias,
               c10::optional<torch::Tensor> resid, torch::Tensor status, c10::optional<torch::Tensor> stamps) {
    c10::cuda::CUDAGuard g(device_);
    const int64_t M = x.size(0);
    const int64_t N = w_mn ? w.size(1) : w.size(0);
    const int64_t need = 2 * M * N * 2;  // two parity halves of W slots of [M/W, N] bf16
    TORCH_CHECK(need <= segs_[staging_].bytes, "staging buffer too small for the fused reduce-scatter");
    CommArgs a = base_args(staging_, 0, x.data_ptr(), out.data_ptr(), M * N, 7, M * N * 2, 1);
    gemm_fused(1, x, w, out, w_mn, bias, c10::nullopt, resid, 0, status, peer_ctx(a), &rs_base_, stamps);
  }

  // out[M, N] = epi(all_gather(x_shard) @ w^T); when given, `gathered` [M, K]
  // receives a copy of the gathered input (copy engine, after the kernel).
  void ag_gemm(torch::Tensor x_shard, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> gathered,
               bool w_mn, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux,
               c10::optional<torch::Tensor> resid, int64_t epi, torch::Tensor status) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(x_shard.is_contiguous() && x_shard.scalar_type() == at::kBFloat16, "x shard: contiguous bf16");
    const int64_t bytes = x_shard.numel() * 2;
    const int64_t full = bytes * world_;
    TORCH_CHECK(2 * full <= segs_[staging_].bytes, "staging buffer too small for the fused all-gather");
    CommArgs a = base_args(staging_, 0, x_shard.data_ptr(), out.data_ptr(), x_shard.numel(), 8, bytes, 1);
    auto stream = at::cuda::getCurrentCUDAStream();
    // Peers' row blocks arrive by push.  My own rows are read in place when
    // they tile evenly (128-row tiles); otherwise they are copied into my block.
    const bool own_in_place = x_shard.size(0) % 128 == 0;
    uint8_t* mine = static_cast<uint8_t*>(a.data[rank_]);
    if (!own_in_place)
      ck(cudaMemcpyAsync(mine + rank_ * bytes, x_shard.data_ptr(), bytes, cudaMemcpyDeviceToDevice, stream),
         "shard copy");
    gemm_fused(2, x_shard, w, out, w_mn, bias, aux, resid, epi, status, peer_ctx(a), &ag_base_, c10::nullopt);
    if (gathered) {
      TORCH_CHECK(gathered->is_contiguous() && gathered->numel() * gathered->element_size() == full,
                  "gathered must be a contiguous [M, K] bf16 tensor");
      uint8_t* g8 = static_cast<uint8_t*>(gathered->data_ptr());
      if (own_in_place) {  // blocks before mine, mine from the input, blocks after mine
        if (rank_ > 0) ck(cudaMemcpyAsync(g8, mine, rank_ * bytes, cudaMemcpyDeviceToDevice, stream), "gathered copy");
        ck(cudaMemcpyAsync(g8 + rank_ * bytes, x_shard.data_ptr(), bytes, cudaMemcpyDeviceToDevice, stream),
           "gathered copy");
        const int64_t after = full - (rank_ + 1) * bytes;
        if (after > 0)
          ck(cudaMemcpyAsync(g8 + (rank_ + 1) * bytes, mine + (rank_ + 1) * bytes, after, cudaMemcpyDeviceToDevice,
                             stream),
             "gathered copy");
      } else {
        ck(cudaMemcpyAsync(g8, mine, full, cudaMemcpyDeviceToDevice, stream), "gathered copy");
      }
    }
  }

  // FSDP: out = x @ W^T (+ bias) with W = rows [0, N) of the weight at
  // w_off in the unit's flat parameter buffer, gathering that buffer from
  // every rank's shard (a symmetric tensor) into `flat` in the same launch.
  void gemm_agw(torch::Tensor x, torch::Tensor shard, torch::Tensor flat, int64_t w_off, int64_t N,
                c10::optional<torch::Tensor> bias, torch::Tensor out, torch::Tensor status) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(shard.is_contiguous() && shard.scalar_type() == at::kBFloat16, "shard: contiguous bf16");
    const int64_t n = shard.numel();
    auto loc = locate(shard.data_ptr(), n * 2);
    TORCH_CHECK(loc.first >= 0, "the shard must be a symmetric tensor of this communicator");
    std::vector<const void*> shards(world_);
    for (int r = 0; r < world_; ++r)
      shards[r] = static_cast<const uint8_t*>(segs_[loc.first].peers[r]) + loc.second;
    if (!agw_cnt_.defined())
      agw_cnt_ = torch::zeros({kMaxRanks * 16 + 1}, torch::TensorOptions().dtype(torch::kInt).device(torch::kCUDA, device_));
    CommArgs a = base_args(staging_, 0, x.data_ptr(), out.data_ptr(), n * world_, 10, n * world_ * 2, 1);
    mnb::gemm_agw(x, flat, w_off, N, bias, out, shards, n, agw_cnt_, status, peer_ctx(a), &ag_base_);
  }

  // shard of sum_r(grad_r) * scale fed straight into AdamW on this rank's shard
  void reduce_scatter_adamw(torch::Tensor grad, torch::Tensor param, c10::optional<torch::Tensor> master,
                            torch::Tensor m, torch::Tensor v, double lr, double b1, double b2, double eps, double wd,
                            double bc1, double bc2, double scale, int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(grad.is_contiguous() && param.is_contiguous(), "contiguous grad and param shard");
    const int64_t n = grad.numel();
    TORCH_CHECK(n % world_ == 0, "gradient length must divide by world size");
    const int64_t chunk = n / world_;
    TORCH_CHECK(param.numel() == chunk && m.numel() == chunk && v.numel() == chunk, "shard sizes disagree");
    TORCH_CHECK(m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat, "moments must be fp32");
    const auto gt = grad.scalar_type();
    TORCH_CHECK(gt == at::kBFloat16 || gt == at::kFloat, "gradient must be bf16 or fp32");
    const auto pt = param.scalar_type();
    TORCH_CHECK(pt == at::kBFloat16 || pt == at::kFloat, "parameters must be bf16 or fp32");
    TORCH_CHECK(staging_need(2, n, grad.element_size()) <= segs_[staging_].bytes, "staging buffer too small");
    CommArgs a = base_args(staging_, 0, grad.data_ptr(), param.data_ptr(), chunk, 9, n * grad.element_size(), 1);
    a.scale = static_cast<float>(scale);
    AdamArgs o{};
    if (master) {
      TORCH_CHECK(master->scalar_type() == at::kFloat && master->numel() == chunk, "master must be fp32 [shard]");
      o.master = master->data_ptr<float>();
    }
    o.m = m.data_ptr<float>();
    o.v = v.data_ptr<float>();
    o.param = param.data_ptr();
    o.lr = static_cast<float>(lr);
    o.b1 = static_cast<float>(b1);
    o.b2 = static_cast<float>(b2);
    o.eps = static_cast<float>(eps);
    o.wd = static_cast<float>(wd);
    o.c1 = static_cast<float>(1.0 / bc1);
    o.c2 = static_cast<float>(1.0 / bc2);
    const int blocks = blocks_for(chunk * grad.element_size(), max_blocks);
    auto stream = at::cuda::getCurrentCUDAStream();
    if (gt == at::kBFloat16) {
      if (pt == at::kBFloat16) rs_adamw_kernel<__nv_bfloat16, true><<<blocks, kCommThreads, 0, stream>>>(a, o);
      else rs_adamw_kernel<__nv_bfloat16, false><<<blocks, kCommThreads, 0, stream>>>(a, o);
    } else {
      if (pt == at::kBFloat16) rs_adamw_kernel<float, true><<<blocks, kCommThreads, 0, stream>>>(a, o);
      else rs_adamw_kernel<float, false><<<blocks, kCommThreads, 0, stream>>>(a, o);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  // algorithm: 0 one_shot, 1 two_shot
  // max_blocks < 0: two-shot sums run as -max_blocks (at most) small CTAs that
  // fit beside a persistent GEMM CTA on one SM (for all-reduces overlapped
  // with compute).  Every rank must pass the same value.
  void all_reduce(torch::Tensor in, torch::Tensor out, int op, int algorithm, int wire_bf16, double scale,
                  int max_blocks) {
    const bool beside = max_blocks < 0;
    if (beside) max_blocks = -max_blocks;
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous() && in.numel() == out.numel(), "contiguous, same size");
    const auto dt = in.scalar_type();
    const int64_t n = in.numel();
    const int64_t wsz = wire_bf16 ? 2 : in.element_size();
    TORCH_CHECK(staging_need(algorithm, n, wsz) <= segs_[staging_].bytes, "staging buffer too small");
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), n, 0, n * wsz, 2);
    a.scale = static_cast<float>(scale);
    if (algorithm == 1 && in.data_ptr() == out.data_ptr()) {
      // in place on a symmetric tensor: results go straight into every rank's copy
      auto loc = locate(in.data_ptr(), n * in.element_size());
      if (loc.first >= 0) {
        const Segment& sg = segs_[loc.first];
        for (int r = 0; r < world_; ++r) a.dst[r] = static_cast<uint8_t*>(sg.peers[r]) + loc.second;
      }
    }
    const int64_t V = 16 / wsz;
    const long long chunk_u = ((n / V) + world_ - 1) / world_;
    const int64_t n_pad = (n + V - 1) / V * V;
    const int64_t per_rank = algorithm == 1 ? n * wsz / world_ : n * wsz;
    auto stream = at::cuda::getCurrentCUDAStream();
    if (beside && algorithm == 1 && op == kSum && (dt == at::kBFloat16 || dt == at::kFloat)) {
      const int nb = blocks_for(per_rank, max_blocks, 16 << 10);
      if (dt == at::kBFloat16)
        ar_push_two_shot_kernel<__nv_bfloat16, __nv_bfloat16, kSum, 128, 6><<<nb, 128, 0, stream>>>(a, chunk_u);
      else if (wire_bf16)
        ar_push_two_shot_kernel<float, __nv_bfloat16, kSum, 128, 6><<<nb, 128, 0, stream>>>(a, chunk_u);
      else
        ar_push_two_shot_kernel<float, float, kSum, 128, 6><<<nb, 128, 0, stream>>>(a, chunk_u);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      return;
    }
    const int blocks = blocks_for(per_rank, max_blocks);
#define MNB_AR1(TI, TW, OPV)                                                                         \
  do {                                                                                              \
    if (algorithm) ar_push_two_shot_kernel<TI, TW, OPV><<<blocks, kCommThreads, 0, stream>>>(a, chunk_u); \
    else ar_push_one_shot_kernel<TI, TW, OPV><<<blocks, kCommThreads, 0, stream>>>(a, n_pad);       \
  } while (0)
#define MNB_AR(TI, TW)                          \
  do {                                         \
    switch (op) {                              \
      case kSum: MNB_AR1(TI, TW, kSum); break;  \
      case kProd: MNB_AR1(TI, TW, kProd); break; \
      case kMax: MNB_AR1(TI, TW, kMax); break;  \
      default: MNB_AR1(TI, TW, kMin); break;    \
    }                                          \
  } while (0)
    if (dt == at::kFloat && wire_bf16) MNB_AR(float, __nv_bfloat16);
    else if (dt == at::kFloat) MNB_AR(float, float);
    else if (dt == at::kBFloat16) MNB_AR(__nv_bfloat16, __nv_bfloat16);
    else if (dt == at::kHalf) MNB_AR(__half, __half);
    else if (dt == at::kLong) MNB_AR(int64_t, int64_t);
    else if (dt == at::kInt) MNB_AR(int32_t, int32_t);
    else TORCH_CHECK(false, "unsupported dtype for device all_reduce");
#undef MNB_AR
#undef MNB_AR1
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  void reduce_scatter(torch::Tensor in, torch::Tensor out, int op, double scale, int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
    const int64_t chunk = out.numel();
    TORCH_CHECK(in.numel() == chunk * world_, "input must hold world_size chunks");
    const auto dt = in.scalar_type();
    const int64_t bytes = in.numel() * in.element_size();
    TORCH_CHECK(staging_need(2, in.numel(), in.element_size()) <= segs_[staging_].bytes, "staging buffer too small");
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), chunk, 1, bytes, 1);
    a.scale = static_cast<float>(scale);
    const int blocks = blocks_for(chunk * in.element_size(), max_blocks);
    auto stream = at::cuda::getCurrentCUDAStream();
#define MNB_RS(T)                                                                                   \
  do {                                                                                             \
    switch (op) {                                                                                  \
      case kSum: reduce_scatter_kernel<T, T, kSum><<<blocks, kCommThreads, 0, stream>>>(a); break;  \
      case kProd: reduce_scatter_kernel<T, T, kProd><<<blocks, kCommThreads, 0, stream>>>(a); break; \
      case kMax: reduce_scatter_kernel<T, T, kMax><<<blocks, kCommThreads, 0, stream>>>(a); break;  \
      default: reduce_scatter_kernel<T, T, kMin><<<blocks, kCommThreads, 0, stream>>>(a); break;    \
    }                                                                                              \
  } while (0)
    if (dt == at::kFloat) MNB_RS(float);
    else if (dt == at::kBFloat16) MNB_RS(__nv_bfloat16);
    else if (dt == at::kHalf) MNB_RS(__half);
    else if (dt == at::kLong) MNB_RS(int64_t);
    else if (dt == at::kInt) MNB_RS(int32_t);
    else TORCH_CHECK(false, "unsupported dtype for device reduce_scatter");
#undef MNB_RS
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  // kind: 0 all_gather (in = shard, out = W shards), 1 broadcast, 2 all_to_all
  void move(torch::Tensor in, torch::Tensor out, int kind, int root, int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
    const int64_t in_bytes = in.numel() * in.element_size();
    const int64_t nb = kind == 2 ? in_bytes / world_ : in_bytes;
    TORCH_CHECK(staging_need(kind == 1 ? 4 : 3, nb, 1) <= segs_[staging_].bytes, "staging buffer too small");
    const bool scatter_gather = kind == 1 && world_ >= 4;
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), nb, 2 + kind, in_bytes, scatter_gather ? 2 : 1);
    a.root = root;
    if (scatter_gather) {
      const int blocks = blocks_for(nb / world_, max_blocks);
      bcast_scatter_gather_kernel<<<blocks, kCommThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
    } else {
      const int blocks = blocks_for(nb, max_blocks);
      move_kernel<<<blocks, kCommThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a, kind);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  void barrier() {
    c10::cuda::CUDAGuard g(device_);
    CommArgs a = base_args(staging_, 0, nullptr, nullptr, 0, 5, 0, 1);
    barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  // Parity schedules; `steps` int64 [S, 5] on the device.
  void stepped_all_reduce(torch::Tensor in, torch::Tensor out, torch::Tensor steps, int op, int round_bf16,
                          double scale) {
    c10::cuda::CUDAGuard g(device_);
    const auto dt = in.scalar_type();
    const int64_t n = in.numel();
    const int n_steps = static_cast<int>(steps.size(0));
    const bool narrow_in = dt == at::kBFloat16 || dt == at::kHalf;
    const int64_t work_elem = (narrow_in && round_bf16) ? 4 : in.element_size();
    TORCH_CHECK(staging_need(5, n, work_elem) <= segs_[staging_].bytes, "message larger than the staging buffer");
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), n, 6, n * (round_bf16 ? 2 : in.element_size()),
                           n_steps + 3);
    a.scale = static_cast<float>(scale);
    const long long* sp = reinterpret_cast<const long long*>(steps.data_ptr<int64_t>());
    int round = round_bf16;
    int dev_blocks = 0;
    cudaDeviceGetAttribute(&dev_blocks, cudaDevAttrMultiProcessorCount, device_);
    const int blocks = std::max(1, std::min<int>(dev_blocks / 2, static_cast<int>((n + 4095) / 4096)));
    auto stream = at::cuda::getCurrentCUDAStream();
    auto launch = [&](auto kern) {
      void* params[] = {&a, const_cast<long long**>(&sp), const_cast<int*>(&n_steps), &round};
      ck(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kern), dim3(blocks), dim3(kCommThreads), params, 0,
                                     stream),
         "cooperative launch");
    };
#define MNB_ST(TI, TK)                                                        \
  do {                                                                       \
    switch (op) {                                                            \
      case kSum: launch(stepped_kernel<TI, TK, kSum>); break;                 \
      case kProd: launch(stepped_kernel<TI, TK, kProd>); break;               \
      case kMax: launch(stepped_kernel<TI, TK, kMax>); break;                 \
      default: launch(stepped_kernel<TI, TK, kMin>); break;                   \
    }                                                                        \
  } while (0)
    if (dt == at::kFloat) MNB_ST(float, float);
    else if (dt == at::kBFloat16 && round_bf16) MNB_ST(__nv_bfloat16, float);
    else if (dt == at::kBFloat16) MNB_ST(__nv_bfloat16, __nv_bfloat16);
    else if (dt == at::kHalf) MNB_ST(__half, __half);
    else if (dt == at::kLong) MNB_ST(int64_t, int64_t);
    else if (dt == at::kInt) MNB_ST(int32_t, int32_t);
    else TORCH_CHECK(false, "unsupported dtype for device all_reduce");
#undef MNB_ST
  }


  // ---- NVLS multicast objects (collective set-up driven from Python) --------
  std::string nvls_reason() const { return nvls_unsupported_reason(device_); }
  int nvls_create(int64_t bytes) {
    c10::cuda::CUDAGuard g(device_);
    nvls_.push_back(std::make_unique<NvlsObject>(rank_, world_, device_, bytes));
    return static_cast<int>(nvls_.size()) - 1;
  }
  py::bytes nvls_socket_name(int id) { return py::bytes(nvls_.at(id)->socket_name()); }
  void nvls_exchange(int id, std::vector<std::string> names, double timeout_s) {
    c10::cuda::CUDAGuard g(device_);
    nvls_.at(id)->exchange(names, timeout_s);
  }
  void nvls_bind(int id) {
    c10::cuda::CUDAGuard g(device_);
    nvls_.at(id)->bind_and_map();
  }
  // Every rank's kernels on the object must have finished (the caller
  // synchronises all ranks first).
  void nvls_release(int id) {
    c10::cuda::CUDAGuard g(device_);
    cudaDeviceSynchronize();
    nvls_.at(id)->release();
    if (nvls_staging_ == id) nvls_staging_ = -1;
  }
  int64_t nvls_bytes(int id) { return nvls_.at(id)->bytes(); }
  void set_nvls_staging(int id) {
    TORCH_CHECK(id >= 0 && id < static_cast<int>(nvls_.size()) && nvls_[id]->mapped(), "bad NVLS staging object");
    nvls_staging_ = id;
  }
  torch::Tensor nvls_tensor(int id, int64_t numel, at::ScalarType dtype) {
    const NvlsObject& o = *nvls_.at(id);
    TORCH_CHECK(o.mapped(), "NVLS object not mapped");
    TORCH_CHECK(numel * static_cast<int64_t>(c10::elementSize(dtype)) <= o.bytes(), "NVLS object too small");
    auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device_);
    return torch::from_blob(o.uc(), {numel}, [](void*) {}, opts);
  }
  std::pair<int, int64_t> locate_nvls(const void* p, int64_t bytes) const {
    const auto a = reinterpret_cast<uintptr_t>(p);
    for (size_t i = 0; i < nvls_.size(); ++i) {
      if (!nvls_[i]->mapped()) continue;
      const auto b = reinterpret_cast<uintptr_t>(nvls_[i]->uc());
      if (a >= b && a + bytes <= b + nvls_[i]->bytes()) return {static_cast<int>(i), static_cast<int64_t>(a - b)};
    }
    return {-1, 0};
  }
  bool is_nvls(torch::Tensor t) {
    return locate_nvls(t.data_ptr(), (t.numel() * t.element_size() + 15) / 16 * 16).first >= 0;
  }

  struct NvlsRegion {
    char* uc;
    char* mc;
    bool staged;
  };
  // The call's region: the tensor itself when it lives (16-byte aligned) in an
  // NVLS object and in-place use is allowed, else this call's parity half of
  // the NVLS staging object.
  NvlsRegion nvls_region(const CommArgs& a, const void* p, int64_t bytes, int64_t need, bool in_place_ok) {
    if (in_place_ok) {
      auto loc = locate_nvls(p, bytes);
      if (loc.first >= 0 && loc.second % 16 == 0) {
        const NvlsObject& o = *nvls_[loc.first];
        return {static_cast<char*>(o.uc()) + loc.second, static_cast<char*>(o.mc()) + loc.second, false};
      }
    }
    TORCH_CHECK(nvls_staging_ >= 0, "NVLS staging buffer not set up");
    const NvlsObject& o = *nvls_[nvls_staging_];
    const int64_t half = (o.bytes() / 2) / 256 * 256;
    TORCH_CHECK(need <= half, "NVLS staging buffer too small for this message");
    const int64_t off = static_cast<int64_t>(a.seq & 1) * half;
    return {static_cast<char*>(o.uc()) + off, static_cast<char*>(o.mc()) + off, true};
  }
  int64_t nvls_staging_half() const {
    return nvls_staging_ < 0 ? 0 : (nvls_[nvls_staging_]->bytes() / 2) / 256 * 256;
  }

  // Sum all-reduce through the switch.  max_blocks < 0: 128-thread CTAs that
  // fit beside a persistent GEMM / attention CTA (all-reduces overlapped with
  // compute); every rank must pass the same value.
  void nvls_all_reduce(torch::Tensor in, torch::Tensor out, double scale, int max_blocks) {
    const bool beside = max_blocks < 0;
    if (beside) max_blocks = -max_blocks;
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous() && in.numel() == out.numel(), "contiguous, same size");
    const auto dt = in.scalar_type();
    TORCH_CHECK(dt == at::kFloat || dt == at::kBFloat16 || dt == at::kHalf, "NVLS all-reduce: fp32, bf16 or fp16");
    const int64_t n = in.numel();
    const int64_t bytes = (n * in.element_size() + 15) / 16 * 16;
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), n, 0, n * in.element_size(), 2);
    a.scale = static_cast<float>(scale);
    const NvlsRegion rg = nvls_region(a, in.data_ptr(), bytes, bytes, in.data_ptr() == out.data_ptr());
    auto stream = at::cuda::getCurrentCUDAStream();
    const int staged = rg.staged ? 1 : 0;
    if (beside) {
      const int nb = blocks_for(bytes / world_, max_blocks, 16 << 10);
      if (dt == at::kFloat) nvls_all_reduce_kernel<float, 128, 6><<<nb, 128, 0, stream>>>(a, rg.uc, rg.mc, staged);
      else if (dt == at::kBFloat16)
        nvls_all_reduce_kernel<__nv_bfloat16, 128, 6><<<nb, 128, 0, stream>>>(a, rg.uc, rg.mc, staged);
      else nvls_all_reduce_kernel<__half, 128, 6><<<nb, 128, 0, stream>>>(a, rg.uc, rg.mc, staged);
    } else {
      const int nb = blocks_for(bytes / world_, max_blocks);
      if (dt == at::kFloat)
        nvls_all_reduce_kernel<float, kCommThreads, 1><<<nb, kCommThreads, 0, stream>>>(a, rg.uc, rg.mc, staged);
      else if (dt == at::kBFloat16)
        nvls_all_reduce_kernel<__nv_bfloat16, kCommThreads, 1><<<nb, kCommThreads, 0, stream>>>(a, rg.uc, rg.mc,
                                                                                                staged);
      else nvls_all_reduce_kernel<__half, kCommThreads, 1><<<nb, kCommThreads, 0, stream>>>(a, rg.uc, rg.mc, staged);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  void nvls_reduce_scatter(torch::Tensor in, torch::Tensor out, double scale, int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
    const auto dt = in.scalar_type();
    TORCH_CHECK(dt == at::kFloat || dt == at::kBFloat16 || dt == at::kHalf, "NVLS reduce-scatter: fp32, bf16 or fp16");
    const int64_t chunk = out.numel();
    TORCH_CHECK(in.numel() == chunk * world_ && (chunk * in.element_size()) % 16 == 0,
                "NVLS reduce-scatter: W chunks of a 16-byte multiple");
    const int64_t bytes = in.numel() * in.element_size();
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), chunk, 1, bytes, 2);
    a.scale = static_cast<float>(scale);
    const NvlsRegion rg = nvls_region(a, in.data_ptr(), bytes, bytes, true);
    const int nb = blocks_for(bytes / world_, max_blocks);
    auto stream = at::cuda::getCurrentCUDAStream();
    const int staged = rg.staged ? 1 : 0;
    if (dt == at::kFloat) nvls_reduce_scatter_kernel<float><<<nb, kCommThreads, 0, stream>>>(a, rg.uc, rg.mc, staged);
    else if (dt == at::kBFloat16)
      nvls_reduce_scatter_kernel<__nv_bfloat16><<<nb, kCommThreads, 0, stream>>>(a, rg.uc, rg.mc, staged);
    else nvls_reduce_scatter_kernel<__half><<<nb, kCommThreads, 0, stream>>>(a, rg.uc, rg.mc, staged);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  // kind 0 all-gather (in = shard, out = W shards), 1 broadcast from `root`.
  void nvls_move(torch::Tensor in, torch::Tensor out, int kind, int root, int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
    const int64_t nb = in.numel() * in.element_size();
    TORCH_CHECK(nb % 16 == 0, "NVLS all-gather / broadcast: a 16-byte multiple per rank");
    const int64_t need = kind == 0 ? nb * world_ : nb;
    TORCH_CHECK(out.numel() * out.element_size() == need, "output size does not match");
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), nb, 2 + kind, need, 2);
    a.root = root;
    const NvlsRegion rg = nvls_region(a, nullptr, 0, need, false);
    const int blocks = blocks_for(nb, max_blocks);
    nvls_move_kernel<<<blocks, kCommThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a, rg.uc, rg.mc, kind);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  void nvls_rs_adamw(torch::Tensor grad, torch::Tensor param, c10::optional<torch::Tensor> master, torch::Tensor m,
                     torch::Tensor v, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                     double scale, int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(grad.is_contiguous() && param.is_contiguous(), "contiguous grad and param shard");
    const int64_t n = grad.numel();
    const int64_t chunk = n / world_;
    TORCH_CHECK(n % world_ == 0 && (chunk * grad.element_size()) % 16 == 0, "NVLS: chunks of a 16-byte multiple");
    TORCH_CHECK(param.numel() == chunk && m.numel() == chunk && v.numel() == chunk, "shard sizes disagree");
    const auto gt = grad.scalar_type(), pt = param.scalar_type();
    TORCH_CHECK(gt == at::kBFloat16 || gt == at::kFloat, "gradient must be bf16 or fp32");
    TORCH_CHECK(pt == at::kBFloat16 || pt == at::kFloat, "parameters must be bf16 or fp32");
    const int64_t bytes = n * grad.element_size();
    CommArgs a = base_args(staging_, 0, grad.data_ptr(), param.data_ptr(), chunk, 9, bytes, 2);
    a.scale = static_cast<float>(scale);
    AdamArgs o{};
    if (master) o.master = master->data_ptr<float>();
    o.m = m.data_ptr<float>();
    o.v = v.data_ptr<float>();
    o.param = param.data_ptr();
    o.lr = static_cast<float>(lr);
    o.b1 = static_cast<float>(b1);
    o.b2 = static_cast<float>(b2);
    o.eps = static_cast<float>(eps);
    o.wd = static_cast<float>(wd);
    o.c1 = static_cast<float>(1.0 / bc1);
    o.c2 = static_cast<float>(1.0 / bc2);
    const NvlsRegion rg = nvls_region(a, grad.data_ptr(), bytes, bytes, true);
    const int blocks = blocks_for(bytes / world_, max_blocks);
    auto stream = at::cuda::getCurrentCUDAStream();
    const int staged = rg.staged ? 1 : 0;
    if (gt == at::kBFloat16) {
      if (pt == at::kBFloat16)
        nvls_rs_adamw_kernel<__nv_bfloat16, true><<<blocks, kCommThreads, 0, stream>>>(a, o, rg.uc, rg.mc, staged);
      else nvls_rs_adamw_kernel<__nv_bfloat16, false><<<blocks, kCommThreads, 0, stream>>>(a, o, rg.uc, rg.mc, staged);
    } else {
      if (pt == at::kBFloat16)
        nvls_rs_adamw_kernel<float, true><<<blocks, kCommThreads, 0, stream>>>(a, o, rg.uc, rg.mc, staged);
      else nvls_rs_adamw_kernel<float, false><<<blocks, kCommThreads, 0, stream>>>(a, o, rg.uc, rg.mc, staged);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  // DDP bucket with the optimizer inside its reduction: reduce `grad`, apply
  // AdamW to this rank's 1/W slice (fp32 master / m / v hold that slice) and
  // write the new parameters into every rank's `param` bucket.  Both buckets
  // are NVLS tensors (switch reduction, multicast store) or peer-mapped
  // symmetric tensors (push kernel).  max_blocks < 0: 128-thread CTAs that
  // fit beside compute.
  void all_reduce_adamw(torch::Tensor grad, torch::Tensor param, torch::Tensor master, torch::Tensor m,
                        torch::Tensor v, double lr, double b1, double b2, double eps, double wd, double bc1,
                        double bc2, double scale, int max_blocks) {
    const bool beside = max_blocks < 0;
    if (beside) max_blocks = -max_blocks;
    c10::cuda::CUDAGuard g(device_);
    const auto dt = grad.scalar_type();
    TORCH_CHECK(dt == param.scalar_type() && (dt == at::kBFloat16 || dt == at::kFloat),
                "gradient and parameter buckets: both bf16 or both fp32");
    TORCH_CHECK(grad.is_contiguous() && param.is_contiguous() && grad.numel() == param.numel(), "bucket shapes");
    const int64_t V = 16 / grad.element_size();
    const int64_t n = grad.numel();
    TORCH_CHECK(n % (world_ * V) == 0, "bucket length must be a multiple of world_size x 16 bytes");
    const int64_t slice = n / world_;
    for (const torch::Tensor* t : {&master, &m, &v})
      TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == slice,
                  "master / m / v: fp32 [bucket / world_size]");
    const int64_t bytes = n * grad.element_size();
    CommArgs a = base_args(staging_, 0, grad.data_ptr(), param.data_ptr(), slice, 11, bytes, 2);
    a.scale = static_cast<float>(scale);
    AdamArgs o{};
    o.master = master.data_ptr<float>();
    o.m = m.data_ptr<float>();
    o.v = v.data_ptr<float>();
    o.param = param.data_ptr();
    o.lr = static_cast<float>(lr);
    o.b1 = static_cast<float>(b1);
    o.b2 = static_cast<float>(b2);
    o.eps = static_cast<float>(eps);
    o.wd = static_cast<float>(wd);
    o.c1 = static_cast<float>(1.0 / bc1);
    o.c2 = static_cast<float>(1.0 / bc2);
    auto stream = at::cuda::getCurrentCUDAStream();
    const int threads = beside ? 128 : kCommThreads;
    const int nb = blocks_for(bytes / world_, max_blocks, beside ? (8 << 10) : (32 << 10));
    const auto lg = locate_nvls(grad.data_ptr(), bytes), lp = locate_nvls(param.data_ptr(), bytes);
    if (lg.first >= 0 && lp.first >= 0 && lg.second % 16 == 0 && lp.second % 16 == 0) {
      char* gmc = static_cast<char*>(nvls_[lg.first]->mc()) + lg.second;
      char* pmc = static_cast<char*>(nvls_[lp.first]->mc()) + lp.second;
#define MNB_NA(T)                                                                                     \
  if (beside) nvls_ar_adamw_kernel<T, 128, 6><<<nb, threads, 0, stream>>>(a, o, gmc, pmc);            \
  else nvls_ar_adamw_kernel<T, kCommThreads, 1><<<nb, threads, 0, stream>>>(a, o, gmc, pmc);
      if (dt == at::kBFloat16) { MNB_NA(__nv_bfloat16) } else { MNB_NA(float) }
#undef MNB_NA
    } else {
      const auto sg = locate(grad.data_ptr(), bytes), spm = locate(param.data_ptr(), bytes);
      TORCH_CHECK(sg.first >= 0 && spm.first >= 0, "both buckets must be symmetric tensors of this communicator");
      TORCH_CHECK(bytes <= (segs_[staging_].bytes / 2) / 256 * 256, "staging buffer too small for the bucket");
      for (int r = 0; r < world_; ++r) a.dst[r] = static_cast<uint8_t*>(segs_[spm.first].peers[r]) + spm.second;
#define MNB_PA(T)                                                                                     \
  if (beside) ar_adamw_push_kernel<T, 128, 6><<<nb, threads, 0, stream>>>(a, o);                      \
  else ar_adamw_push_kernel<T, kCommThreads, 1><<<nb, threads, 0, stream>>>(a, o);
      if (dt == at::kBFloat16) { MNB_PA(__nv_bfloat16) } else { MNB_PA(float) }
#undef MNB_PA
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  int rank() const { return rank_; }
  int world() const { return world_; }

 private:
  int rank_, world_, device_;
  void* sig_local_ = nullptr;
  std::vector<uint32_t*> sig_peers_;
  bool sig_opened_ = false;
  std::vector<Segment> segs_;
  int staging_ = 0;
  volatile int* status_h_ = nullptr;
  volatile int* status_d_ = nullptr;
  DevEvent* ring_h_ = nullptr;
  DevEvent* ring_d_ = nullptr;
  uint32_t epoch_ = 1;
  uint32_t ag_base_ = 0;  // total arrival-counter increments of fused all-gathers so far
  uint32_t rs_base_ = 0;  // ... and of fused reduce-scatters
  uint32_t seq_ = 0;
  unsigned long long timeout_ns_ = 300ull * 1000000000ull;
  bool closed_ = false;
  std::vector<std::unique_ptr<NvlsObject>> nvls_;
  int nvls_staging_ = -1;
  torch::Tensor agw_cnt_;  // chunk counters of the FSDP gather-GEMM (zeroed per launch)
};

void register_comm(py::module_& m) {
  py::class_<DeviceCommImpl>(m, "DeviceCommImpl")
      .def(py::init<int, int, int, int64_t>())
      .def("add_segment", &DeviceCommImpl::add_segment)
      .def("segment_handle", &DeviceCommImpl::segment_handle)
      .def("signal_handle", &DeviceCommImpl::signal_handle)
      .def("open_segment", &DeviceCommImpl::open_segment)
      .def("open_signals", &DeviceCommImpl::open_signals)
      .def("segment_ptr", &DeviceCommImpl::segment_ptr)
      .def("segment_bytes", &DeviceCommImpl::segment_bytes)
      .def("staging_segment", &DeviceCommImpl::staging_segment)
      .def("set_staging", &DeviceCommImpl::set_staging)
      .def("segment_tensor", &DeviceCommImpl::segment_tensor)
      .def("is_symmetric", &DeviceCommImpl::is_symmetric)
      .def("status", &DeviceCommImpl::status)
      .def("clear_status", &DeviceCommImpl::clear_status)
      .def("set_timeout", &DeviceCommImpl::set_timeout)
      .def("seq", &DeviceCommImpl::seq)
      .def("events", &DeviceCommImpl::events)
      .def("all_reduce", &DeviceCommImpl::all_reduce)
      .def("reduce_scatter", &DeviceCommImpl::reduce_scatter)
      .def("move", &DeviceCommImpl::move)
      .def("barrier", &DeviceCommImpl::barrier)
      .def("stepped_all_reduce", &DeviceCommImpl::stepped_all_reduce)
      .def("staging_need", &DeviceCommImpl::staging_need)
      .def("gemm_rs", &DeviceCommImpl::gemm_rs)
      .def("reduce_scatter_adamw", &DeviceCommImpl::reduce_scatter_adamw)
      .def("ag_gemm", &DeviceCommImpl::ag_gemm)
      .def("gemm_agw", &DeviceCommImpl::gemm_agw)
      .def("nvls_reason", &DeviceCommImpl::nvls_reason)
      .def("nvls_create", &DeviceCommImpl::nvls_create)
      .def("nvls_socket_name", &DeviceCommImpl::nvls_socket_name)
      .def("nvls_exchange", &DeviceCommImpl::nvls_exchange)
      .def("nvls_bind", &DeviceCommImpl::nvls_bind)
      .def("nvls_release", &DeviceCommImpl::nvls_release)
      .def("nvls_bytes", &DeviceCommImpl::nvls_bytes)
      .def("set_nvls_staging", &DeviceCommImpl::set_nvls_staging)
      .def("nvls_staging_half", &DeviceCommImpl::nvls_staging_half)
      .def("nvls_tensor", &DeviceCommImpl::nvls_tensor)
      .def("is_nvls", &DeviceCommImpl::is_nvls)
      .def("nvls_all_reduce", &DeviceCommImpl::nvls_all_reduce)
      .def("nvls_reduce_scatter", &DeviceCommImpl::nvls_reduce_scatter)
      .def("nvls_move", &DeviceCommImpl::nvls_move)
      .def("nvls_rs_adamw", &DeviceCommImpl::nvls_rs_adamw)
      .def("all_reduce_adamw", &DeviceCommImpl::all_reduce_adamw)
      .def("close", &DeviceCommImpl::close)
      .def_property_readonly("rank", &DeviceCommImpl::rank)
      .def_property_readonly("world", &DeviceCommImpl::world);
}

}  // namespace mnb
