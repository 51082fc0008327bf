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
#include <string>
#include <vector>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace mnb {

constexpr int kMaxRanks = 16;
constexpr int kMaxBlocks = 64;
constexpr int kCommThreads = 512;
constexpr int kSigSlots = kMaxBlocks * kMaxRanks;
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
  void* data[kMaxRanks];     // per-rank peer-visible buffer for this call
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

// ---------------------------------------------------------------------------
// one-shot all-reduce
// ---------------------------------------------------------------------------
template <typename TI, typename TW, int OP>
__global__ void __launch_bounds__(kCommThreads) ar_one_shot_kernel(CommArgs a) {
  using TA = typename Acc<TW>::type;
  constexpr int V = Vec<TW>::n;
  ring_begin(a);
  const long long nu = a.n / V;
  const long long tail = a.n - nu * V;
  long long lo, hi;
  block_range(nu, &lo, &hi);
  if (a.copy_in) {
    copy_in_units<TI, TW>(a, lo, hi);
    if (blockIdx.x == 0 && threadIdx.x < tail) {
      reinterpret_cast<TW*>(a.data[a.rank])[nu * V + threadIdx.x] =
          narrow<TW, TA>(widen<TA, TI>(reinterpret_cast<const TI*>(a.in)[nu * V + threadIdx.x]));
    }
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  if (ok) {
    TI* out = reinterpret_cast<TI*>(a.out);
    for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
      TA acc[V], v[V];
      load_vec<TW, TA>(reinterpret_cast<const TW*>(a.data[0]) + u * V, acc);
      for (int p = 1; p < a.world; ++p) {
        load_vec<TW, TA>(reinterpret_cast<const TW*>(a.data[p]) + u * V, v);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = combine<OP>(acc[i], v[i]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc[i], a.scale)));
      store_out<TI, TA, V>(out + u * V, acc);
    }
    if (blockIdx.x == 0 && threadIdx.x < tail) {
      const long long e = nu * V + threadIdx.x;
      TA acc = widen<TA, TW>(reinterpret_cast<const TW*>(a.data[0])[e]);
      for (int p = 1; p < a.world; ++p) acc = combine<OP>(acc, widen<TA, TW>(reinterpret_cast<const TW*>(a.data[p])[e]));
      out[e] = narrow<TI, TA>(widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc, a.scale))));
    }
    ok = peer_barrier(a, a.epoch + 2);
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// two-shot all-reduce (reduce-scatter + all-gather), in place on symmetric data
// ---------------------------------------------------------------------------
template <typename TI, typename TW, int OP>
__global__ void __launch_bounds__(kCommThreads) ar_two_shot_kernel(CommArgs a) {
  using TA = typename Acc<TW>::type;
  constexpr int V = Vec<TW>::n;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long nu = a.n / V;
  const long long tail = a.n - nu * V;
  const long long cu = (nu + W - 1) / W;  // units per rank chunk
  const long long sub = (cu + gridDim.x - 1) / gridDim.x;
  auto sub_range = [&](int c, long long* lo, long long* hi) {
    const long long c0 = min(nu, c * cu), c1 = min(nu, c0 + cu);
    *lo = min(c1, c0 + sub * blockIdx.x);
    *hi = min(c1, *lo + sub);
  };
  if (a.copy_in) {
    for (int c = 0; c < W; ++c) {
      long long lo, hi;
      sub_range(c, &lo, &hi);
      copy_in_units<TI, TW>(a, lo, hi);
    }
    if (blockIdx.x == 0 && threadIdx.x < tail) {
      reinterpret_cast<TW*>(a.data[r])[nu * V + threadIdx.x] =
          narrow<TW, TA>(widen<TA, TI>(reinterpret_cast<const TI*>(a.in)[nu * V + threadIdx.x]));
    }
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  TI* out = reinterpret_cast<TI*>(a.out);
  TW* mine = reinterpret_cast<TW*>(a.data[r]);
  TA tail_val = 0;
  if (ok) {
    long long lo, hi;
    sub_range(r, &lo, &hi);
    for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
      TA acc[V], v[V];
      load_vec<TW, TA>(reinterpret_cast<const TW*>(a.data[0]) + u * V, acc);
      for (int p = 1; p < W; ++p) {
        load_vec<TW, TA>(reinterpret_cast<const TW*>(a.data[p]) + u * V, v);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = combine<OP>(acc[i], v[i]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = finish<OP>(acc[i], a.scale);
      store_vec<TW, TA>(mine + u * V, acc);  // publish the reduced chunk (wire type)
      TA back[V];
#pragma unroll
      for (int i = 0; i < V; ++i) back[i] = widen<TA, TW>(narrow<TW, TA>(acc[i]));
      if (static_cast<const void*>(out) != static_cast<const void*>(mine)) store_out<TI, TA, V>(out + u * V, back);
    }
    if (blockIdx.x == 0 && threadIdx.x < tail) {
      const long long e = nu * V + threadIdx.x;
      TA acc = widen<TA, TW>(reinterpret_cast<const TW*>(a.data[0])[e]);
      for (int p = 1; p < W; ++p) acc = combine<OP>(acc, widen<TA, TW>(reinterpret_cast<const TW*>(a.data[p])[e]));
      tail_val = widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc, a.scale)));
    }
    ok = peer_barrier(a, a.epoch + 2);
  }
  if (ok) {
    for (int c = 0; c < W; ++c) {
      if (c == r) continue;
      long long lo, hi;
      sub_range(c, &lo, &hi);
      for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
        TA v[V];
        load_vec<TW, TA>(reinterpret_cast<const TW*>(a.data[c]) + u * V, v);
        store_out<TI, TA, V>(out + u * V, v);
      }
    }
    ok = peer_barrier(a, a.epoch + 3);
    // the tail is written last: it may live inside `mine`, which peers read until the barrier above
    if (ok && blockIdx.x == 0 && threadIdx.x < tail) out[nu * V + threadIdx.x] = narrow<TI, TA>(tail_val);
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// reduce-scatter: out[chunk] = scale * reduce_p in_p[rank*chunk : (rank+1)*chunk]
// ---------------------------------------------------------------------------
template <typename TI, typename TW, int OP>
__global__ void __launch_bounds__(kCommThreads) reduce_scatter_kernel(CommArgs a) {
  using TA = typename Acc<TW>::type;
  constexpr int V = Vec<TW>::n;
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long chunk = a.n;
  const bool vec = chunk % V == 0;
  if (a.copy_in) {
    const long long total = chunk * W;
    long long lo, hi;
    block_range(total, &lo, &hi);
    const TI* in = reinterpret_cast<const TI*>(a.in);
    TW* w = reinterpret_cast<TW*>(a.data[r]);
    for (long long e = lo + threadIdx.x; e < hi; e += blockDim.x) w[e] = narrow<TW, TA>(widen<TA, TI>(in[e]));
  }
  // The copy-in partition (whole message) differs from the reduce partition
  // (my chunk), so every block must finish staging before any peer reads:
  // barrier across all blocks of all ranks via block 0's slots is not enough,
  // hence a grid-uniform partition -- every block staged a slice of the whole
  // message and waits for *every* block index of every peer below.
  bool ok = peer_barrier(a, a.epoch + 1);
  if (ok && a.copy_in) {
    // wait until all peers' other blocks have staged too: poll their slots for all block ids
    const int t = threadIdx.x;
    if (t < a.world * gridDim.x) {
      const int p = t % a.world, blk = t / a.world;
      if (p != r) {
        const uint32_t* slot = a.sig[r] + blk * kMaxRanks + p;
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (static_cast<int32_t>(ld_acquire_sys(slot) - (a.epoch + 1)) < 0) {
          if ((++spins & 255u) == 0) {
            if (a.status[0] != 0 || globaltimer_ns() - t0 > a.timeout_ns) {
              if (a.status[0] == 0) {
                a.status[1] = p; a.status[2] = blk; a.status[3] = static_cast<int>(a.seq);
                __threadfence_system();
                a.status[0] = kErrPeerTimeout;
              }
              break;
            }
            __nanosleep(64);
          }
        }
      }
    }
    ok = __syncthreads_and(a.status[0] == 0) != 0;
  }
  if (ok) {
    TI* out = reinterpret_cast<TI*>(a.out);
    if (vec) {
      long long lo, hi;
      block_range(chunk / V, &lo, &hi);
      for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
        TA acc[V], v[V];
        const long long off = r * chunk + u * V;
        load_vec<TW, TA>(reinterpret_cast<const TW*>(a.data[0]) + off, acc);
        for (int p = 1; p < W; ++p) {
          load_vec<TW, TA>(reinterpret_cast<const TW*>(a.data[p]) + off, v);
#pragma unroll
          for (int i = 0; i < V; ++i) acc[i] = combine<OP>(acc[i], v[i]);
        }
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc[i], a.scale)));
        store_out<TI, TA, V>(out + u * V, acc);
      }
    } else {
      long long lo, hi;
      block_range(chunk, &lo, &hi);
      for (long long e = lo + threadIdx.x; e < hi; e += blockDim.x) {
        const long long off = r * chunk + e;
        TA acc = widen<TA, TW>(reinterpret_cast<const TW*>(a.data[0])[off]);
        for (int p = 1; p < W; ++p) acc = combine<OP>(acc, widen<TA, TW>(reinterpret_cast<const TW*>(a.data[p])[off]));
        out[e] = narrow<TI, TA>(widen<TA, TW>(narrow<TW, TA>(finish<OP>(acc, a.scale))));
      }
    }
    ok = peer_barrier(a, a.epoch + 2);
  }
  ring_end(a, ok);
}

// ---------------------------------------------------------------------------
// data movement without reduction (byte-level): all-gather, broadcast, all-to-all
//   kind 0 all_gather: out[p*chunk + e] = data[p][e]
//   kind 1 broadcast : out[e] = data[root][e]
//   kind 2 all_to_all: out[p*chunk + e] = data[p][rank*chunk + e]
// sizes in bytes (n = per-rank chunk bytes for 0/2, message bytes for 1)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCommThreads) move_kernel(CommArgs a, int kind, long long in_bytes) {
  ring_begin(a);
  const int W = a.world, r = a.rank;
  const long long nb = a.n;
  if (a.copy_in) {
    const bool stage = kind != 1 || r == a.root;
    if (stage) {
      long long lo, hi;
      const bool v16 = in_bytes % 16 == 0;
      const long long units = v16 ? in_bytes / 16 : in_bytes;
      block_range(units, &lo, &hi);
      for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
        if (v16) st_v4(reinterpret_cast<uint8_t*>(a.data[r]) + 16 * u, ld_v4(reinterpret_cast<const uint8_t*>(a.in) + 16 * u));
        else reinterpret_cast<uint8_t*>(a.data[r])[u] = reinterpret_cast<const uint8_t*>(a.in)[u];
      }
    }
  }
  bool ok = peer_barrier(a, a.epoch + 1);
  // staging partition (bytes of the input) can differ from the read partition; wait for all block ids
  if (ok && a.copy_in) {
    const int t = threadIdx.x;
    if (t < W * gridDim.x) {
      const int p = t % W, blk = t / W;
      if (p != r) {
        const uint32_t* slot = a.sig[r] + blk * kMaxRanks + p;
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (static_cast<int32_t>(ld_acquire_sys(slot) - (a.epoch + 1)) < 0) {
          if ((++spins & 255u) == 0) {
            if (a.status[0] != 0 || globaltimer_ns() - t0 > a.timeout_ns) {
              if (a.status[0] == 0) {
                a.status[1] = p; a.status[2] = blk; a.status[3] = static_cast<int>(a.seq);
                __threadfence_system();
                a.status[0] = kErrPeerTimeout;
              }
              break;
            }
            __nanosleep(64);
          }
        }
      }
    }
    ok = __syncthreads_and(a.status[0] == 0) != 0;
  }
  if (ok) {
    const bool v16 = nb % 16 == 0 && (kind != 2 || (static_cast<long long>(r) * nb) % 16 == 0);
    const long long units = v16 ? nb / 16 : nb;
    long long lo, hi;
    block_range(units, &lo, &hi);
    uint8_t* out = reinterpret_cast<uint8_t*>(a.out);
    for (int p = 0; p < W; ++p) {
      const uint8_t* src;
      uint8_t* dst;
      if (kind == 0) {
        src = reinterpret_cast<const uint8_t*>(a.data[p]);
        dst = out + p * nb;
      } else if (kind == 1) {
        if (p != 0) break;
        if (r == a.root && a.out == a.in) break;
        src = reinterpret_cast<const uint8_t*>(a.data[a.root]);
        dst = out;
      } else {
        src = reinterpret_cast<const uint8_t*>(a.data[p]) + r * nb;
        dst = out + p * nb;
      }
      for (long long u = lo + threadIdx.x; u < hi; u += blockDim.x) {
        if (v16) st_v4(dst + 16 * u, ld_v4_volatile(src + 16 * u));
        else dst[u] = src[u];
      }
    }
    ok = peer_barrier(a, a.epoch + 2);
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
    for (int r = 0; r < world_; ++r) {
      a.data[r] = static_cast<uint8_t*>(s.peers[r]) + offset;
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

  int blocks_for(int64_t bytes, int max_blocks) const {
    int64_t b = (bytes + (256 << 10) - 1) / (256 << 10);  // ~256 KiB per CTA
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(b, std::min(max_blocks, kMaxBlocks))));
  }

  // algorithm: 0 one_shot, 1 two_shot
  void all_reduce(torch::Tensor in, torch::Tensor out, int op, int algorithm, int wire_bf16, double scale,
                  int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous() && in.numel() == out.numel(), "contiguous, same size");
    const auto dt = in.scalar_type();
    const int64_t n = in.numel();
    const int64_t wsz = wire_bf16 ? 2 : in.element_size();
    auto loc = locate(in.data_ptr(), n * in.element_size());
    const bool zero_copy = algorithm == 1 && !wire_bf16 && loc.first >= 0 && in.data_ptr() == out.data_ptr();
    int seg = staging_;
    int64_t off = 0;
    if (zero_copy) {
      seg = loc.first;
      off = loc.second;
    } else {
      TORCH_CHECK(n * wsz <= segs_[staging_].bytes, "message larger than the staging buffer");
    }
    CommArgs a = base_args(seg, off, in.data_ptr(), out.data_ptr(), n, 0, n * wsz, 3);
    a.scale = static_cast<float>(scale);
    a.copy_in = zero_copy ? 0 : 1;
    const int blocks = blocks_for(n * wsz / std::max(1, algorithm == 1 ? 1 : 1), max_blocks);
    auto stream = at::cuda::getCurrentCUDAStream();
#define MNB_AR(TI, TW)                                                                              \
  do {                                                                                             \
    switch (op) {                                                                                  \
      case kSum: (algorithm ? ar_two_shot_kernel<TI, TW, kSum> : ar_one_shot_kernel<TI, TW, kSum>)  \
          <<<blocks, kCommThreads, 0, stream>>>(a); break;                                          \
      case kProd: (algorithm ? ar_two_shot_kernel<TI, TW, kProd> : ar_one_shot_kernel<TI, TW, kProd>) \
          <<<blocks, kCommThreads, 0, stream>>>(a); break;                                          \
      case kMax: (algorithm ? ar_two_shot_kernel<TI, TW, kMax> : ar_one_shot_kernel<TI, TW, kMax>)  \
          <<<blocks, kCommThreads, 0, stream>>>(a); break;                                          \
      default: (algorithm ? ar_two_shot_kernel<TI, TW, kMin> : ar_one_shot_kernel<TI, TW, kMin>)    \
          <<<blocks, kCommThreads, 0, stream>>>(a); break;                                          \
    }                                                                                              \
  } while (0)
    if (dt == at::kFloat && wire_bf16) MNB_AR(float, __nv_bfloat16);
    else if (dt == at::kFloat) MNB_AR(float, float);
    else if (dt == at::kBFloat16) MNB_AR(__nv_bfloat16, __nv_bfloat16);
    else if (dt == at::kHalf) MNB_AR(__half, __half);
    else if (dt == at::kLong) MNB_AR(int64_t, int64_t);
    else if (dt == at::kInt) MNB_AR(int32_t, int32_t);
    else TORCH_CHECK(false, "unsupported dtype for device all_reduce");
#undef MNB_AR
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }

  void reduce_scatter(torch::Tensor in, torch::Tensor out, int op, double scale, int max_blocks) {
    c10::cuda::CUDAGuard g(device_);
    TORCH_CHECK(in.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
    const int64_t chunk = out.numel();
    TORCH_CHECK(in.numel() == chunk * world_, "input must hold world_size chunks");
    const auto dt = in.scalar_type();
    const int64_t bytes = in.numel() * in.element_size();
    auto loc = locate(in.data_ptr(), bytes);
    int seg = staging_;
    int64_t off = 0;
    if (loc.first >= 0) {
      seg = loc.first;
      off = loc.second;
    } else {
      TORCH_CHECK(bytes <= segs_[staging_].bytes, "message larger than the staging buffer");
    }
    CommArgs a = base_args(seg, off, in.data_ptr(), out.data_ptr(), chunk, 1, bytes, 2);
    a.scale = static_cast<float>(scale);
    a.copy_in = loc.first >= 0 ? 0 : 1;
    const int blocks = blocks_for(chunk * in.element_size() * world_, max_blocks);
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
    const int64_t nb = kind == 0 ? in_bytes : (kind == 1 ? in_bytes : in_bytes / world_);
    auto loc = locate(in.data_ptr(), in_bytes);
    int seg = staging_;
    int64_t off = 0;
    if (loc.first >= 0) {
      seg = loc.first;
      off = loc.second;
    } else {
      TORCH_CHECK(in_bytes <= segs_[staging_].bytes, "message larger than the staging buffer");
    }
    CommArgs a = base_args(seg, off, in.data_ptr(), out.data_ptr(), nb, 2 + kind, in_bytes, 2);
    a.root = root;
    a.copy_in = loc.first >= 0 ? 0 : 1;
    const int blocks = blocks_for(kind == 1 ? in_bytes : in_bytes * world_, max_blocks);
    move_kernel<<<blocks, kCommThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a, kind, in_bytes);
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
    TORCH_CHECK(n * work_elem <= segs_[staging_].bytes, "message larger than the staging buffer");
    CommArgs a = base_args(staging_, 0, in.data_ptr(), out.data_ptr(), n, 6, n * (round_bf16 ? 2 : in.element_size()),
                           n_steps + 2);
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
  uint32_t seq_ = 0;
  unsigned long long timeout_ns_ = 300ull * 1000000000ull;
  bool closed_ = false;
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
      .def("close", &DeviceCommImpl::close)
      .def_property_readonly("rank", &DeviceCommImpl::rank)
      .def_property_readonly("world", &DeviceCommImpl::world);
}

}  // namespace mnb
