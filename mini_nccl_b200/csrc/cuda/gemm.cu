// tcgen05 GEMM for sm_100a: D = A * B^T with fused epilogues.
//
// Layout (M, N, K logical):
//   A is [M, K] K-major (row-major, K contiguous), or with a_mn [K, M] (M contiguous)
//   B is [N, K] K-major, or with b_mn [K, N] (N contiguous)
// which covers every GEMM of a linear layer:
//   forward   Y  = X  W^T : A = X  (K-major), B = W (K-major)
//   data grad dX = dY W   : A = dY (K-major), B = W stored [N_out, K_in] -> MN-major
//   weight    dW = dY^T X : A = dY stored [tokens, N] -> MN-major,
//                           B = X  stored [tokens, K] -> MN-major
//
// Kernel structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: one elected lane streams 128x64 A and BNx64 B
//               tiles (128-byte swizzle) into a STAGES-deep ring of shared
//               memory, each slot guarded by a full/empty mbarrier pair.
//   warp 1      owns the TMEM allocation (2 x BN fp32 columns: double-buffered
//               accumulators) and one lane issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction) and tcgen05.commit to release smem slots
//               and to publish a finished accumulator.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each thread owns one row),
//               apply bias / GELU / residual / accumulate, convert, store.
//               While they drain accumulator i the MMA warp fills accumulator
//               i^1 for the next tile.
// TMA loads are per-CTA (no cluster multicast).  Every wait is bounded and
// reports through args.status instead of hanging.
//
// Fused with a collective (tensor parallelism with a sequence-parallel
// layout; the ranks of one device communicator run the same launch):
//   kFuseRS  GEMM -> reduce-scatter.  Every rank computes partial sums for all
//            M rows; the epilogue stores each finished tile straight into the
//            staging slot of the rank that owns those rows (NVLink stores from
//            registers), so the transfer of tile i overlaps the MMAs of tile
//            i+1.  Tiles are visited starting with the next rank's rows and
//            ending with this rank's own.  When a CTA has no tiles left it
//            signals every owner; once all CTAs of all ranks have signalled,
//            the CTAs sum the W slots of this rank's rows in rank order and
//            add bias and residual (bf16 out).
//   kFuseAG  all-gather -> GEMM.  The gathered A is this call's staging
//            region ([M, K], row block s = rank s's shard, own block copied in
//            by the copy engine before the launch).  Two extra warps per CTA
//            push this CTA's slice of the own shard into every peer's staging
//            (16-byte coalesced NVLink stores) and then bump the peer's
//            arrival counter for this source with a release atomic; the TMA
//            producer waits for a shard's counter before loading its rows.
//            Tiles of the own rows come first, so the exchange runs under
//            them; every remote row crosses NVLink once and the TMA unit only
//            reads local memory.
//   kFuseAGW all-gather of the weight -> GEMM (FSDP).  B is a weight inside
//            a flattened parameter buffer that every rank holds one shard of.
//            Two extra warps per CTA first meet every other rank's CTAs (so
//            no shard is read before its owner has entered the collective),
//            then claim parts of chunks from one work counter -- the chunks
//            that hold this GEMM's weight first, in row order, then the rest
//            of the buffer -- and copy them from the owner's shard (peer
//            loads) into the local gathered buffer, counting every copied part
//            on its chunk.  The TMA producer waits only for the chunks that
//            hold the B rows of its tile, so the first tiles start after the
//            first chunks arrive and the rest of the gather runs under the
//            MMAs.  When the launch ends the whole buffer is gathered (the
//            unit's later GEMMs read it).  Parts are claimed dynamically, so
//            progress never depends on one particular CTA being resident.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <cstdlib>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "peer.cuh"

namespace mnb {

enum : int {
  kEpiNone = 0,
  kEpiBias = 1,       // + bias[col]
  kEpiGelu = 2,       // out = gelu(acc + bias), aux = acc + bias (pre-activation)
  kEpiResid = 4,      // + resid[row, col]
  kEpiGeluGrad = 8,   // out = acc * gelu'(aux[row, col])
  kEpiAccum = 16,     // out += acc (read-modify-write of the existing output)
  kEpiOutF32 = 32,    // fp32 output instead of bf16
};

struct GemmArgs {
  int M, N, K;
  int k_blocks_per_split;
  int splits;
  void* out;
  long long ldo;
  long long split_stride;  // elements between split-K partial outputs (fp32 workspace)
  const __nv_bfloat16* bias;
  __nv_bfloat16* aux;
  long long ldaux;
  const __nv_bfloat16* resid;
  long long ldr;
  int epi;
  int tma_out;  // bf16 output (and GELU aux) written through shared memory + TMA store
  int red_out;  // split-K: fp32 partial tiles added into one workspace by TMA reduce-add
  int* status;
  // fused collectives
  int rows_per_rank;                // M / world (RS: rows each rank owns; AG: rows of each shard)
  const __nv_bfloat16* ag_local;    // AG: this rank's shard of A, [rows_per_rank, K]
  uint32_t ag_target;               // AG: counter value meaning "every CTA of that rank has pushed"
  uint32_t rs_target;               // RS: counter value meaning "every CTA of that rank has stored its tiles"
  int ag_own_map;                   // AG: own rows are read through map_own from the input (rows % 128 == 0)
  unsigned long long* stamps;       // optional %globaltimer phase stamps (CTA 0 / slowest CTA), or null
  // kFuseAGW: B = rows of a weight inside the gathered flat parameter buffer
  const __nv_bfloat16* agw_src[kMaxRanks];  // every rank's shard (peer addresses; own = local)
  __nv_bfloat16* agw_flat;                  // local gathered buffer [world * agw_shard]
  long long agw_shard;                      // shard elements (multiple of 8)
  long long agw_chunk;                      // chunk elements (multiple of 8)
  long long agw_w_off;                      // flat offset of B's row 0 (B is [N, K], row stride K)
  long long agw_bias_off;                   // flat offset of the bias, or -1
  int agw_nch;                              // chunks per shard
  int agw_parts;                            // parts per chunk (the unit of claimed work)
  int agw_pri_first, agw_pri_last;          // chunk range holding B (and its bias): gathered first
  uint32_t* agw_cnt;                        // [world * nch] per-chunk part counts, then the work counter
  int agw_shallow;                          // 8 loads in flight per gather thread instead of 16 (A/B)
};

enum : int { kFuseNone = 0, kFuseRS = 1, kFuseAG = 2, kFuseAGW = 3 };

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quadrant, each owning half the columns
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kGatherThreads = 64;  // kFuseAG: two gather warps after the epilogue warps
template <int FUSE>
constexpr int gemm_threads() { return kGemmThreads + ((FUSE == kFuseAG || FUSE == kFuseAGW) ? kGatherThreads : 0); }

MNB_DEVICE uint32_t ld_acquire_gpu(const int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
MNB_DEVICE void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MNB_DEVICE void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// 16-byte load that bypasses L1 (another GPU's memory, rewritten between launches).
MNB_DEVICE uint4 ld_v4_cg_peer(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Output tile visiting order.  RS: start with the next rank's rows and end
// with our own (their transfer is local); AG: our own rows first (no wait).
template <int FUSE>
MNB_DEVICE int remap_mblock(int mb, int m_tiles, const GemmArgs& a, const PeerCtx& ctx) {
  if constexpr (FUSE == kFuseNone || FUSE == kFuseAGW) {
    return mb;
  } else {
    if (a.rows_per_rank % kBM != 0) return mb;
    const int per = a.rows_per_rank / kBM;
    const int first = FUSE == kFuseRS ? (ctx.rank + 1) % ctx.world : ctx.rank;
    return (mb + first * per) % m_tiles;
  }
}

// RS epilogue: a staged 32-row x 64-column bf16 box (128-byte swizzle) goes
// to the owners' slots for this rank; lane l moves 16-byte chunk l%8 of rows
// l/8, l/8+4, ...
MNB_DEVICE void rs_push_box(const GemmArgs& a, const PeerCtx& ctx, const uint8_t* box, int row0, int col0,
                            int lane) {
  const int chunk = lane & 7;
  const int col = col0 + chunk * 8;
  if (col >= a.N) return;  // N is a multiple of 8: a chunk is all in or all out
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int rr = it * 4 + (lane >> 3);
    const int row = row0 + rr;
    if (row >= a.M) break;
    const uint4 val = *reinterpret_cast<const uint4*>(box + rr * 128 + ((chunk ^ (rr & 7)) * 16));
    const int o = row / a.rows_per_rank;
    const long long lr = row - static_cast<long long>(o) * a.rows_per_rank;
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ctx.data[o]) +
                       (static_cast<long long>(ctx.rank) * a.rows_per_rank + lr) * a.N + col;
    st_v4(d, val);
  }
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr uint32_t a_bytes = kBM * kBK * 2;
  static constexpr uint32_t b_bytes = BN * kBK * 2;
  static constexpr uint32_t ring = STAGES * (a_bytes + b_bytes);
  // 32-row x 128-byte staging boxes per epilogue warp: two (output + GELU aux)
  // in the 3-stage configuration, one in the 4-stage configuration
  static constexpr uint32_t boxes = STAGES <= 3 ? 2 : 1;
  static constexpr uint32_t staging = 8 * boxes * 4096;
  static constexpr uint32_t bars = (2 * STAGES + 4) * 8;
  static constexpr uint32_t total = ring + staging + bars + 16 + 1024;  // + tmem slot + alignment slack
};

MNB_DEVICE void epilogue_store(const GemmArgs& a, int row, int col0, float* v) {
  const int N = a.N;
  if (row >= a.M) return;
  const bool full = col0 + 32 <= N;
  if (a.epi & kEpiBias) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      int c = col0 + i;
      v[i] += (c < N) ? bf16_to_f32(a.bias[c]) : 0.f;
    }
  }
  if (a.epi & kEpiGelu) {
    __nv_bfloat16* ap = a.aux + static_cast<long long>(row) * a.ldaux + col0;
    if (full) {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        st_v4(ap + 8 * i, make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]));
    } else {
      _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) ap[i] = f32_to_bf16(v[i]);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_exact(v[i]);
  }
  if (a.epi & kEpiGeluGrad) {
    const __nv_bfloat16* ap = a.aux + static_cast<long long>(row) * a.ldaux + col0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 w = ld_v4(ap + 8 * i);
        uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = unpack_bf16x2(ws[j]);
          v[8 * i + 2 * j] *= gelu_grad(f.x);
          v[8 * i + 2 * j + 1] *= gelu_grad(f.y);
        }
      }
    } else {
      _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) v[i] *= gelu_grad(bf16_to_f32(ap[i]));
    }
  }
  if (a.epi & kEpiResid) {
    const __nv_bfloat16* rp = a.resid + static_cast<long long>(row) * a.ldr + col0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 w = ld_v4(rp + 8 * i);
        uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = unpack_bf16x2(ws[j]);
          v[8 * i + 2 * j] += f.x;
          v[8 * i + 2 * j + 1] += f.y;
        }
      }
    } else {
      _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) v[i] += bf16_to_f32(rp[i]);
    }
  }
  if (a.epi & kEpiOutF32) {
    float* op = reinterpret_cast<float*>(a.out) + static_cast<long long>(row) * a.ldo + col0;
    if (full) {
      if (a.epi & kEpiAccum) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 o = reinterpret_cast<float4*>(op)[i];
          v[4 * i] += o.x; v[4 * i + 1] += o.y; v[4 * i + 2] += o.z; v[4 * i + 3] += o.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(op)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
      _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) op[i] = (a.epi & kEpiAccum) ? op[i] + v[i] : v[i];
    }
    return;
  }
  __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + static_cast<long long>(row) * a.ldo + col0;
  if (full) {
    if (a.epi & kEpiAccum) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 w = ld_v4(op + 8 * i);
        uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = unpack_bf16x2(ws[j]);
          v[8 * i + 2 * j] += f.x;
          v[8 * i + 2 * j + 1] += f.y;
        }
      }
    }
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      st_v4(op + 8 * i, make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]));
  } else {
    _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) {
      float x = v[i];
      if (a.epi & kEpiAccum) x += bf16_to_f32(op[i]);
      op[i] = f32_to_bf16(x);
    }
  }
}

// Write 32 bf16 values (one row segment) as 16-byte chunks sub*4.. of a
// 32-row x 128-byte box laid out in the 128-byte swizzle (conflict-free).
// 32 floats -> row `row` of a 32-row x 128-byte fp32 staging box (128-byte swizzle)
MNB_DEVICE void stage_row_f32(uint8_t* box, int row, const float* v) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    *reinterpret_cast<float4*>(box + row * 128 + ((k ^ (row & 7)) * 16)) =
        make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

MNB_DEVICE void stage_row32(uint8_t* box, int row, int sub, const float* v) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int chunk = sub * 4 + k;
    *reinterpret_cast<uint4*>(box + row * 128 + ((chunk ^ (row & 7)) * 16)) =
        make_uint4(pack_bf16x2(v[8 * k], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                   pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
  }
}

// Bias / GELU' / residual on 32 consecutive columns of one row (no stores).
MNB_DEVICE void epilogue_inputs(const GemmArgs& a, int row, int col0, float* v) {
  const int N = a.N;
  const bool in_rows = row < a.M;
  const bool full = col0 + 32 <= N;
  if (a.epi & kEpiBias) {
    if (full) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 w = ld_v4(a.bias + col0 + 8 * i);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(ws[j]);
          v[8 * i + 2 * j] += f.x;
          v[8 * i + 2 * j + 1] += f.y;
        }
      }
    } else {
      _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) v[i] += bf16_to_f32(a.bias[col0 + i]);
    }
  }
  if ((a.epi & kEpiGeluGrad) && in_rows) {
    const __nv_bfloat16* ap = a.aux + static_cast<long long>(row) * a.ldaux + col0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 w = ld_v4(ap + 8 * i);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(ws[j]);
          v[8 * i + 2 * j] *= gelu_grad(f.x);
          v[8 * i + 2 * j + 1] *= gelu_grad(f.y);
        }
      }
    } else {
      _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) v[i] *= gelu_grad(bf16_to_f32(ap[i]));
    }
  }
  if ((a.epi & kEpiResid) && in_rows) {
    const __nv_bfloat16* rp = a.resid + static_cast<long long>(row) * a.ldr + col0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 w = ld_v4(rp + 8 * i);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(ws[j]);
          v[8 * i + 2 * j] += f.x;
          v[8 * i + 2 * j + 1] += f.y;
        }
      }
    } else {
      _Pragma("unroll") for (int i = 0; i < 32; ++i) if (col0 + i < N) v[i] += bf16_to_f32(rp[i]);
    }
  }
}

// Epilogue inputs without stalls on dependent global loads:
//  * the bias of the warp's BN/2 columns is loaded once per tile, before the
//    accumulator wait, BN/64 values per lane, and broadcast by shuffles;
//  * the per-row input (residual or GELU pre-activation) of chunk k+1 is
//    loaded while chunk k is being processed.
struct EpiPrefetch {
  uint2 bias;     // BN/64 bf16 values of this lane's slice of the warp's columns
  uint4 row[4];   // 32 bf16 of the next chunk's row input
};

template <int BN>
MNB_DEVICE void load_bias_slice(const GemmArgs& a, int colw, int lane, EpiPrefetch& f) {
  constexpr int vpl = BN / 64;  // values per lane (4 or 2)
  const int c = colw + vpl * lane;
  f.bias = make_uint2(0u, 0u);
  if (a.bias == nullptr) return;
  if (vpl == 4) {
    if (c + 4 <= a.N) f.bias = *reinterpret_cast<const uint2*>(a.bias + c);
  } else {
    if (c + 2 <= a.N) f.bias.x = *reinterpret_cast<const uint32_t*>(a.bias + c);
  }
}

MNB_DEVICE const __nv_bfloat16* row_input(const GemmArgs& a, long long row, int col0) {
  if (a.epi & kEpiResid) return a.resid + row * a.ldr + col0;
  return a.aux + row * a.ldaux + col0;
}

MNB_DEVICE void load_row_chunk(const GemmArgs& a, int row, int col0, uint4* dst) {
  if (row < a.M && col0 + 32 <= a.N) {
    const __nv_bfloat16* p = row_input(a, row, col0);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = ld_v4(p + 8 * i);
  }
}

// bias (shuffled) + row input (prefetched) on 32 values of warp-local chunk k
template <int BN>
MNB_DEVICE void apply_inputs_fast(const GemmArgs& a, const EpiPrefetch& f, int k, const uint4* rowv, float* v) {
  constexpr int vpl = BN / 64;
  if (a.epi & kEpiBias) {
#pragma unroll
    for (int jp = 0; jp < 16; ++jp) {
      const int c = 32 * k + 2 * jp;
      const uint32_t word = ((c % vpl) / 2 == 0) ? f.bias.x : f.bias.y;
      const float2 b2 = unpack_bf16x2(__shfl_sync(0xffffffffu, word, c / vpl));
      const float2 r = add2(make_float2(v[2 * jp], v[2 * jp + 1]), b2);
      v[2 * jp] = r.x;
      v[2 * jp + 1] = r.y;
    }
  }
  if (a.epi & (kEpiResid | kEpiGeluGrad)) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t ws[4] = {rowv[i].x, rowv[i].y, rowv[i].z, rowv[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = unpack_bf16x2(ws[j]);
        const float2 cur = make_float2(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
        const float2 r = (a.epi & kEpiResid) ? add2(cur, x) : mul2(cur, gelu_grad2(x));
        v[8 * i + 2 * j] = r.x;
        v[8 * i + 2 * j + 1] = r.y;
      }
    }
  }
}

// kFuseAG exchange warps (64 threads): push this CTA's slice of the own
// shard into every peer's staging, then count the arrival there.
MNB_DEVICE void push_shard(const GemmArgs& a, const PeerCtx& ctx, int gt) {
  const int W = ctx.world, r = ctx.rank;
  const long long row_units = a.K / 8;  // 16-byte units per row
  const long long rpr = a.rows_per_rank;
  const long long per = (rpr + gridDim.x - 1) / gridDim.x;
  const long long lo = min(rpr, per * static_cast<long long>(blockIdx.x));
  const long long hi = min(rpr, lo + per);
  const long long units = (hi - lo) * row_units;
  const __nv_bfloat16* s0 = a.ag_local + lo * a.K;
  const long long dst_off = (static_cast<long long>(r) * rpr + lo) * a.K;  // own block in everyone's staging
  constexpr int U = 8;
  for (long long u0 = gt; u0 < units; u0 += U * kGatherThreads) {
    uint4 v[U];
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (u0 + j * kGatherThreads < units) v[j] = ld_v4(s0 + 8 * (u0 + j * kGatherThreads));
    for (int k = 1; k < W; ++k) {
      __nv_bfloat16* d0 = reinterpret_cast<__nv_bfloat16*>(ctx.data[(r + k) % W]) + dst_off;
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (u0 + j * kGatherThreads < units) st_v4(d0 + 8 * (u0 + j * kGatherThreads), v[j]);
    }
  }
  asm volatile("bar.sync 2, %0;" ::"n"(kGatherThreads) : "memory");
  if (gt == 0) {
    __threadfence_system();
    for (int k = 1; k < W; ++k) red_release_sys_add(ctx.sig[(r + k) % W] + kCountRow * kMaxRanks + r, 1u);
  }
}


// ---- kFuseAGW ---------------------------------------------------------------
// Order in which chunks are gathered: the chunks holding B first, in flat
// (= weight row) order, then the chunks before them, then those after them.
MNB_DEVICE int agw_chunk_at(const GemmArgs& a, int o) {
  const int n_pri = a.agw_pri_last - a.agw_pri_first + 1;
  if (o < n_pri) return a.agw_pri_first + o;
  const int q = o - n_pri;
  return q < a.agw_pri_first ? q : q + n_pri;
}

MNB_DEVICE int agw_chunk_of(const GemmArgs& a, long long f) {
  const int s = static_cast<int>(f / a.agw_shard);
  return s * a.agw_nch + static_cast<int>((f - s * a.agw_shard) / a.agw_chunk);
}

// Producer side: wait until every chunk overlapping flat elements [f0, f1) is
// gathered.  Bounded; false on timeout or when another wait already failed.
MNB_DEVICE bool agw_wait_range(const GemmArgs& a, const PeerCtx& ctx, long long f0, long long f1) {
  if (f1 <= f0) return true;
  const int g1 = agw_chunk_of(a, f1 - 1);
  const uint64_t t0 = globaltimer_ns();
  for (int g = agw_chunk_of(a, f0); g <= g1; ++g) {
    const int* c = reinterpret_cast<const int*>(a.agw_cnt + g);
    uint32_t spins = 0;
    while (static_cast<int>(ld_acquire_gpu(c)) < a.agw_parts) {
      if ((++spins & 255u) == 0) {
        if (*reinterpret_cast<volatile int*>(a.status) != 0) return false;
        if (globaltimer_ns() - t0 > ctx.timeout_ns) {
          atomicCAS(a.status, 0, kErrPeerTimeout);
          return false;
        }
        __nanosleep(128);
      }
    }
  }
  return true;
}

// Gather warps (64 threads).
MNB_DEVICE void agw_gather(const GemmArgs& a, const PeerCtx& ctx, int gt) {
  const int W = ctx.world, r = ctx.rank;
  __shared__ int agw_flag;
  if (gt == 0) {
    // Meet every rank: its shard is final once it has entered this launch,
    // and it is only written again after a later collective this rank joins.
    __threadfence_system();
    for (int k = 0; k < W; ++k) red_release_sys_add(ctx.sig[k] + kCountRow * kMaxRanks + r, 1u);
    bool ok = true;
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; ok && p < W; ++p)
      ok = wait_signal(ctx.sig[r] + kCountRow * kMaxRanks + p, a.ag_target, ctx.status, p, blockIdx.x, ctx.seq,
                       ctx.timeout_ns, t0);
    if (!ok) atomicCAS(a.status, 0, kErrPeerTimeout);
    agw_flag = ok ? 1 : 0;
  }
  asm volatile("bar.sync 2, %0;" ::"n"(kGatherThreads) : "memory");
  if (!agw_flag) return;
  const int total = W * a.agw_nch;
  const int claims = total * a.agw_parts;
  for (;;) {
    if (gt == 0) agw_flag = static_cast<int>(atomicAdd(a.agw_cnt + total, 1u));
    asm volatile("bar.sync 2, %0;" ::"n"(kGatherThreads) : "memory");
    const int w = agw_flag;
    if (w >= claims) break;
    const int g = agw_chunk_at(a, w / a.agw_parts), part = w % a.agw_parts;
    const int src = g / a.agw_nch;
    const long long c0 = static_cast<long long>(g % a.agw_nch) * a.agw_chunk;
    const long long c1 = min(a.agw_shard, c0 + a.agw_chunk);
    const long long units = c0 < c1 ? (c1 - c0) / 8 : 0;
    const long long per = (units + a.agw_parts - 1) / a.agw_parts;
    const long long lo = min(units, part * per), hi = min(units, lo + per);
    const __nv_bfloat16* from = a.agw_src[src] + c0;
    __nv_bfloat16* to = a.agw_flat + static_cast<long long>(src) * a.agw_shard + c0;
    // U independent 16-byte peer loads in flight per thread: the gather is
    // bound by NVLink load latency, not by issue (U = 16: 16 KB per CTA)
    auto copy = [&](auto u_const) {
      constexpr int U = decltype(u_const)::value;
      for (long long u0 = lo + gt; u0 < hi; u0 += U * kGatherThreads) {
        uint4 v[U];
#pragma unroll
        for (int j = 0; j < U; ++j)
          if (u0 + j * kGatherThreads < hi) v[j] = ld_v4_cg_peer(from + 8 * (u0 + j * kGatherThreads));
#pragma unroll
        for (int j = 0; j < U; ++j)
          if (u0 + j * kGatherThreads < hi) st_v4(to + 8 * (u0 + j * kGatherThreads), v[j]);
      }
    };
    if (a.agw_shallow) copy(std::integral_constant<int, 8>{});
    else copy(std::integral_constant<int, 16>{});
    asm volatile("bar.sync 2, %0;" ::"n"(kGatherThreads) : "memory");  // part copied; agw_flag free again
    if (gt == 0) {
      __threadfence();
      red_release_gpu_add(reinterpret_cast<int*>(a.agw_cnt + g), 1);
    }
  }
}

// kFuseRS tail (all threads): announce that this CTA's tiles have landed,
// wait for every CTA of every rank, then reduce this rank's rows.
MNB_DEVICE void rs_finish(const GemmArgs& a, const PeerCtx& ctx) {
  const int W = ctx.world, r = ctx.rank;
  __syncthreads();
  // stamps: [1] latest "my tiles are done", [2] latest "all flags seen", [3] latest "reduced"
  if (a.stamps != nullptr && threadIdx.x == 0) atomicMax(a.stamps + 1, globaltimer_ns());
  bool ok = *reinterpret_cast<volatile int*>(a.status) == 0;
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's tile stores are visible before its arrival is
    for (int p = 0; p < W; ++p) red_release_sys_add(ctx.sig[p] + kRsCountRow * kMaxRanks + r, 1u);
    const uint64_t t0 = globaltimer_ns();
    for (int src = 0; ok && src < W; ++src)
      ok = wait_signal(ctx.sig[r] + kRsCountRow * kMaxRanks + src, a.rs_target, ctx.status, src, blockIdx.x,
                       ctx.seq, ctx.timeout_ns, t0);
  }
  if (!__syncthreads_and(ok)) return;
  if (a.stamps != nullptr && threadIdx.x == 0) atomicMax(a.stamps + 2, globaltimer_ns());
  // out[row, col] = bias[col] + resid[row, col] + sum_p slot_p[row, col]   (rows of this rank)
  const long long cu = a.N / 8;
  const long long total = static_cast<long long>(a.rows_per_rank) * cu;
  const long long slot = static_cast<long long>(a.rows_per_rank) * a.N;
  const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(ctx.data[r]);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  const long long nthr = static_cast<long long>(gridDim.x) * blockDim.x;
  constexpr int U = 4;  // independent 16-byte units per thread per pass
  auto add8 = [](float* acc, uint4 w) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(ws[j]);
      acc[2 * j] += f.x;
      acc[2 * j + 1] += f.y;
    }
  };
  for (long long u0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; u0 < total; u0 += U * nthr) {
    float acc[U][8];
#pragma unroll
    for (int k = 0; k < U; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;
    for (int p = 0; p < W; ++p) {  // rank order
      uint4 w[U];
#pragma unroll
      for (int k = 0; k < U; ++k)
        if (u0 + k * nthr < total) w[k] = ld_v4_volatile(base + p * slot + (u0 + k * nthr) * 8);
#pragma unroll
      for (int k = 0; k < U; ++k)
        if (u0 + k * nthr < total) add8(acc[k], w[k]);
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const long long u = u0 + k * nthr;
      if (u >= total) continue;
      const long long row = u / cu, col = (u - row * cu) * 8;
      if (a.bias != nullptr) add8(acc[k], ld_v4(a.bias + col));
      if (a.resid != nullptr) add8(acc[k], ld_v4(a.resid + row * a.ldr + col));
      st_v4(out + row * a.ldo + col,
            make_uint4(pack_bf16x2(acc[k][0], acc[k][1]), pack_bf16x2(acc[k][2], acc[k][3]),
                       pack_bf16x2(acc[k][4], acc[k][5]), pack_bf16x2(acc[k][6], acc[k][7])));
    }
  }
  if (a.stamps != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) atomicMax(a.stamps + 3, globaltimer_ns());
  }
}

template <int BN, bool A_MN, bool B_MN, int STAGES, int FUSE>
__global__ void __launch_bounds__(gemm_threads<FUSE>(), 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_out, const __grid_constant__ CUtensorMap map_aux,
                        const __grid_constant__ CUtensorMap map_own, const GemmArgs args, const PeerCtx ctx) {
  using S = GemmSmem<BN, STAGES>;
  constexpr uint32_t kIdesc = idesc_bf16(kBM, BN, A_MN, B_MN);
  constexpr uint32_t kTmemCols = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ring_a = smem;
  uint8_t* ring_b = smem + STAGES * S::a_bytes;
  uint8_t* staging = smem + S::ring;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::ring + S::staging);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES);
  const uint32_t tempty0 = smem_u32(bars + 2 * STAGES + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(tfull0 + 8 * s, 1);
      mbar_init(tempty0 + 8 * s, 32 * kEpiWarps);
    }
    fence_mbar_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (args.stamps != nullptr && blockIdx.x == 0 && threadIdx.x == 0) args.stamps[0] = globaltimer_ns();

  const int m_tiles = (args.M + kBM - 1) / kBM;
  const int n_tiles = (args.N + BN - 1) / BN;
  const int k_blocks = (args.K + kBK - 1) / kBK;
  const int units = m_tiles * n_tiles * args.splits;
  int* status = args.status;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ready_mask = 0;  // kFuseAG: shards known to be gathered
      (void)ready_mask;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int split = u / (m_tiles * n_tiles);
        const int t = u % (m_tiles * n_tiles);
        const int mb = remap_mblock<FUSE>(t % m_tiles, m_tiles, args, ctx), nb = t / m_tiles;
        const int kb0 = split * args.k_blocks_per_split;
        const int kb1 = min(k_blocks, kb0 + args.k_blocks_per_split);
        bool ok = true;
        if constexpr (FUSE == kFuseAG) {
          // rows of this tile come from shards s0..s1: wait until every CTA
          // of those ranks has pushed its part into this rank's staging
          const int s0 = (mb * kBM) / args.rows_per_rank;
          const int s1 = min(args.M - 1, mb * kBM + kBM - 1) / args.rows_per_rank;
          for (int sh = s0; sh <= s1 && ok; ++sh) {
            if (sh == ctx.rank || (ready_mask & (1u << sh))) continue;
            ok = wait_signal(ctx.sig[ctx.rank] + kCountRow * kMaxRanks + sh, args.ag_target, ctx.status, sh,
                             blockIdx.x, ctx.seq, ctx.timeout_ns, globaltimer_ns());
            if (!ok) atomicCAS(status, 0, kErrPeerTimeout);
            ready_mask |= 1u << sh;
          }
          fence_proxy_async_global();  // generic-proxy (peer) writes -> TMA reads
        }
        if constexpr (FUSE == kFuseAGW) {
          // B rows of this tile (and, before the first tile, the bias the
          // epilogue reads) must have been gathered
          if (u == static_cast<int>(blockIdx.x) && args.agw_bias_off >= 0)
            ok = agw_wait_range(args, ctx, args.agw_bias_off, args.agw_bias_off + args.N);
          const long long r0 = static_cast<long long>(nb) * BN, r1 = min(static_cast<long long>(args.N), r0 + BN);
          if (ok) ok = agw_wait_range(args, ctx, args.agw_w_off + r0 * args.K, args.agw_w_off + r1 * args.K);
          fence_proxy_async_global();  // generic-proxy writes of the gather warps -> TMA reads
        }
        for (int kb = kb0; kb < kb1 && ok; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, status)) { ok = false; break; }
          const uint32_t full = full0 + 8 * stage;
          mbar_arrive_expect_tx(full, S::a_bytes + S::b_bytes);
          const uint32_t sa = smem_u32(ring_a + stage * S::a_bytes);
          const uint32_t sb = smem_u32(ring_b + stage * S::b_bytes);
          const int k0 = kb * kBK;
          if (!A_MN) {
            if (FUSE == kFuseAG && args.ag_own_map && mb * kBM / args.rows_per_rank == ctx.rank)
              tma_load_2d(sa, &map_own, k0, mb * kBM - ctx.rank * args.rows_per_rank, full);  // own rows, in place
            else
              tma_load_2d(sa, &map_a, k0, mb * kBM, full);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j) tma_load_2d(sa + j * 8192, &map_a, mb * kBM + 64 * j, k0, full);
          }
          if (!B_MN) {
            tma_load_2d(sb, &map_b, k0, nb * BN, full);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &map_b, nb * BN + 64 * j, k0, full);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int split = u / (m_tiles * n_tiles);
        const int kb0 = split * args.k_blocks_per_split;
        const int kb1 = min(k_blocks, kb0 + args.k_blocks_per_split);
        if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, status)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase, status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(ring_a + stage * S::a_bytes);
          const uint32_t sb = smem_u32(ring_b + stage * S::b_bytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = A_MN ? smem_desc_sw128(sa + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(sb + k * 2048, 8192, 1024)
                                     : smem_desc_sw128(sb + k * 32, 16, 1024);
            tc_mma(d, ad, bd, kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(empty0 + 8 * stage);  // slot free once these MMAs have read it
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(tfull0 + 8 * acc);  // accumulator ready for the epilogue
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // Epilogue warps 2..9: warp w may only touch TMEM lanes 32*(w%4) .. +31;
    // warps w and w+4 share a quadrant and split its columns in halves.
    const int q = warp & 3;
    const int half = (warp - 2) / 4;
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int split = u / (m_tiles * n_tiles);
      const int t = u % (m_tiles * n_tiles);
      const int mb = remap_mblock<FUSE>(t % m_tiles, m_tiles, args, ctx), nb = t / m_tiles;
      // Fast input path: bf16 TMA-store epilogues with at most one per-row
      // input; its loads are issued before the accumulator wait.
      const bool fast = FUSE != kFuseRS && args.tma_out &&
                        !((args.epi & kEpiResid) && (args.epi & kEpiGeluGrad));
      const bool row_in = (args.epi & (kEpiResid | kEpiGeluGrad)) != 0;
      EpiPrefetch pf;
      if (fast) {
        load_bias_slice<BN>(args, nb * BN + half * (BN / 2), lane, pf);
        if (row_in) load_row_chunk(args, mb * kBM + row_in_tile, nb * BN + half * (BN / 2), pf.row);
      }
      bool ok = mbar_wait(tfull0 + 8 * acc, acc_phase, status);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      GemmArgs a = args;
      if (args.splits > 1)
        a.out = reinterpret_cast<float*>(args.out) + static_cast<long long>(split) * args.split_stride;
      const int row = mb * kBM + row_in_tile;
      const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      bool released = false;  // accumulator handed back early (TMA-store path)
      if (FUSE == kFuseRS) {
        // 32 rows x 64 columns at a time: registers -> swizzled smem box ->
        // 128-byte row segments stored into the owner's slot (a warp store
        // covers four whole segments, the efficient shape for NVLink writes)
        uint8_t* box = staging + (warp - 2) * (S::boxes * 4096);
#pragma unroll 1
        for (int g = half * (BN / 128); g < (half + 1) * (BN / 128); ++g) {
          const int colg = nb * BN + g * 64;
          if (colg >= a.N) break;
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            float v[32];
            tmem_ld_32(lane_addr + g * 64 + sub * 32, v);
            stage_row32(box, lane, sub, v);
          }
          __syncwarp();
          rs_push_box(a, ctx, box, mb * kBM + q * 32, colg, lane);
          __syncwarp();
        }
      } else if (a.tma_out) {
        // 64-column groups: TMEM -> registers -> epilogue math -> swizzled
        // staging box -> one TMA store per 32 x 64 block (rows/cols past the
        // matrix are clipped by the TMA unit).
        uint8_t* box_out = staging + (warp - 2) * (S::boxes * 4096);
        uint8_t* box_aux = box_out + (S::boxes - 1) * 4096;  // == box_out with one box
        const bool gelu = (a.epi & kEpiGelu) != 0;
        const int g_end = (half + 1) * (BN / 128);
#pragma unroll 1
        for (int g = half * (BN / 128); g < g_end; ++g) {
          const int colg = nb * BN + g * 64;
          if (colg >= a.N) break;
          // with two boxes and a single output, alternate them (double buffer)
          uint8_t* bo = (!gelu && S::boxes == 2 && (g & 1)) ? box_aux : box_out;
          float v64[64];
          tmem_ld_64(lane_addr + g * 64, v64);  // both 32-column halves, one wait
          if (g + 1 == g_end || colg + 64 >= a.N) {
            // this warp's last columns are in registers: hand the accumulator
            // back to the MMA warp before the math and the stores
            tc_fence_before();
            mbar_arrive(tempty0 + 8 * acc);
            released = true;
          }
          if (lane == 0) {  // the staging box is free once the previous store has read it
            if (gelu || S::boxes == 1) bulk_wait_read<0>();
            else bulk_wait_read<1>();
          }
          __syncwarp();
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            float* v = v64 + sub * 32;
            const int k = (g - half * (BN / 128)) * 2 + sub;  // warp-local chunk
            const int col0 = colg + sub * 32;
            if (fast && col0 + 32 <= a.N) {
              uint4 cur[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) cur[i] = pf.row[i];
              if (row_in && k + 1 < BN / 64) load_row_chunk(a, row, col0 + 32, pf.row);  // next chunk's input
              apply_inputs_fast<BN>(a, pf, k, cur, v);
            } else {
              epilogue_inputs(a, row, col0, v);
            }
            if (gelu) {
              stage_row32(box_aux, lane, sub, v);  // pre-activation
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float2 g = gelu_exact2(make_float2(v[i], v[i + 1]));
                v[i] = g.x;
                v[i + 1] = g.y;
              }
            }
            stage_row32(bo, lane, sub, v);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_out, smem_u32(bo), colg, mb * kBM + q * 32);
            if (gelu) tma_store_2d(&map_aux, smem_u32(box_aux), colg, mb * kBM + q * 32);
            bulk_commit();
          }
        }
      } else if (a.red_out) {
        // split-K partial sums: 32 x 32 fp32 boxes -> staging -> TMA reduce-add
        // into the one fp32 workspace (the adds run at L2; rows and columns
        // past the matrix are clipped by the TMA unit)
        uint8_t* box = staging + (warp - 2) * (S::boxes * 4096);
        const int c_end = (half + 1) * (BN / 64);
#pragma unroll 1
        for (int c = half * (BN / 64); c < c_end; ++c) {
          const int col0 = nb * BN + c * 32;
          if (col0 >= a.N) break;
          float v[32];
          tmem_ld_32(lane_addr + c * 32, v);
          if (c + 1 == c_end || col0 + 32 >= a.N) {
            tc_fence_before();
            mbar_arrive(tempty0 + 8 * acc);
            released = true;
          }
          if (lane == 0) bulk_wait_read<0>();  // the box is free once the previous reduce has read it
          __syncwarp();
          stage_row_f32(box, lane, v);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&map_out, smem_u32(box), col0, mb * kBM + q * 32);
            bulk_commit();
          }
        }
      } else {
#pragma unroll 1
        for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
          float v[32];
          tmem_ld_32(lane_addr + c * 32, v);
          const int col0 = nb * BN + c * 32;
          if (col0 < a.N) epilogue_store(a, row, col0, v);
        }
      }
      if (!released) {
        tc_fence_before();
        mbar_arrive(tempty0 + 8 * acc);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  } else if constexpr (FUSE == kFuseAG) {
    push_shard(args, ctx, threadIdx.x - kGemmThreads);
  } else if constexpr (FUSE == kFuseAGW) {
    agw_gather(args, ctx, threadIdx.x - kGemmThreads);
  }

  if (warp >= 2 && warp < 2 + kEpiWarps && lane == 0) bulk_wait_all();  // staging boxes drained before exit
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if constexpr (FUSE == kFuseRS) rs_finish(args, ctx);
}

// Sum split-K fp32 partials into the final output (bf16 or fp32), optionally
// accumulating into what is already there.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, long long split_stride,
                                     int M, int N, void* out, long long ldo, int out_f32, int accumulate) {
  const long long total4 = static_cast<long long>(M) * N / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = 4 * i;
    const int row = static_cast<int>(e / N), col = static_cast<int>(e % N);
    float4 s = reinterpret_cast<const float4*>(ws)[i];
    for (int k = 1; k < splits; ++k) {
      float4 p = reinterpret_cast<const float4*>(ws + k * split_stride)[i];
      s.x += p.x; s.y += p.y; s.z += p.z; s.w += p.w;
    }
    if (out_f32) {
      float* o = reinterpret_cast<float*>(out) + row * ldo + col;
      if (accumulate) { s.x += o[0]; s.y += o[1]; s.z += o[2]; s.w += o[3]; }
      *reinterpret_cast<float4*>(o) = s;
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + row * ldo + col;
      if (accumulate) {
        uint2 w = *reinterpret_cast<uint2*>(o);
        float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
        s.x += a.x; s.y += a.y; s.z += b.x; s.w += b.y;
      }
      *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(s.x, s.y), pack_bf16x2(s.z, s.w));
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

CUtensorMap make_tma_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                             uint32_t box_inner, uint32_t box_outer) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(r));
  return map;
}

// fp32 [outer, inner] matrix, 128-byte swizzle: box_inner * 4 must be <= 128.
CUtensorMap make_tma_2d_f32(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                            uint32_t box_inner, uint32_t box_outer) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 4) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TORCH_CHECK(box_inner * 4 <= 128, "128-byte swizzle: inner box of at most 32 floats");
  CUtensorMap map;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp32) failed: ", static_cast<int>(r));
  return map;
}

int num_sms() {
  static int n = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

template <int BN, bool A_MN, bool B_MN, int STAGES, int FUSE = kFuseNone>
void launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const CUtensorMap& mx,
                 const GemmArgs& args, int units, cudaStream_t stream, const PeerCtx& ctx = PeerCtx{},
                 const CUtensorMap* mown = nullptr) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, STAGES, FUSE>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::total));
    configured = true;
  }
  // Fused launches wait on one another across CTAs (and ranks): one CTA per
  // SM at most, so every CTA of the grid is resident at once.
  const int grid = std::min(units, num_sms());
  kern<<<grid, gemm_threads<FUSE>(), S::total, stream>>>(ma, mb, mo, mx, mown ? *mown : ma, args, ctx);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Inner-dim contiguity + 16-byte row strides are what TMA needs.
static int64_t row_stride(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must be contiguous in its last dimension");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0, name, " row stride must be a multiple of 8 elements");
  return t.stride(0);
}

// Public entry: out = epi(A * B^T) with the layouts described at the top.
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool a_mn, bool b_mn,
          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux,
          c10::optional<torch::Tensor> resid, int64_t epi, int64_t splits,
          c10::optional<torch::Tensor> workspace, torch::Tensor status) {
  c10::cuda::CUDAGuard guard(a.device());
  const int64_t lda = row_stride(a, "A");
  const int64_t ldb = row_stride(b, "B");
  const int M = static_cast<int>(a_mn ? a.size(1) : a.size(0));
  const int K = static_cast<int>(a_mn ? a.size(0) : a.size(1));
  const int N = static_cast<int>(b_mn ? b.size(1) : b.size(0));
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "A and B disagree on K");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "bad output shape");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "N and K must be multiples of 8");
  const bool out_f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(out_f32 || out.scalar_type() == at::kBFloat16, "output must be bf16 or fp32");
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  args.epi = static_cast<int>(epi) | (out_f32 ? kEpiOutF32 : 0);
  args.status = status.data_ptr<int>();
  if (bias) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "bias must be bf16 [N]");
    args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
    args.epi |= kEpiBias;
  }
  if (aux) {
    TORCH_CHECK(aux->scalar_type() == at::kBFloat16 && aux->stride(1) == 1, "aux must be bf16 row-major");
    args.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
    args.ldaux = aux->stride(0);
  }
  if (resid) {
    TORCH_CHECK(resid->scalar_type() == at::kBFloat16 && resid->stride(1) == 1, "resid must be bf16 row-major");
    args.resid = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
    args.ldr = resid->stride(0);
    args.epi |= kEpiResid;
  }
  const int k_blocks = (K + kBK - 1) / kBK;
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, k_blocks));
  const int per = static_cast<int>((k_blocks + splits - 1) / splits);
  splits = (k_blocks + per - 1) / per;  // no empty splits
  args.k_blocks_per_split = per;
  args.splits = static_cast<int>(splits);
  if (splits > 1) {
    // every split adds its partial tiles into one zeroed fp32 workspace (TMA
    // reduce-add); a conversion pass writes the output
    TORCH_CHECK(workspace.has_value() && workspace->scalar_type() == at::kFloat && workspace->is_contiguous() &&
                    workspace->numel() >= static_cast<int64_t>(M) * N,
                "split-K needs a contiguous fp32 workspace of M*N");
    TORCH_CHECK(!(args.epi & ~(kEpiAccum | kEpiOutF32)), "split-K supports plain/accumulate epilogues only");
    TORCH_CHECK(N % 4 == 0, "split-K needs N % 4 == 0 (16-byte workspace rows)");
    args.out = workspace->data_ptr();
    args.ldo = N;
    args.split_stride = 0;
    args.epi = kEpiOutF32;
    args.red_out = 1;
  } else {
    args.out = out.data_ptr();
    args.ldo = out.stride(0);
  }
  const bool wide = N >= 256;
  const int BN = wide ? 256 : 128;
  const int m_tiles = (M + kBM - 1) / kBM;
  const int n_tiles = (N + BN - 1) / BN;
  const int units = m_tiles * n_tiles * static_cast<int>(splits);
  CUtensorMap ma = a_mn ? make_tma_2d_bf16(a.data_ptr(), M, K, lda, 64, 64)
                        : make_tma_2d_bf16(a.data_ptr(), K, M, lda, 64, kBM);
  CUtensorMap mb = b_mn ? make_tma_2d_bf16(b.data_ptr(), N, K, ldb, 64, 64)
                        : make_tma_2d_bf16(b.data_ptr(), K, N, ldb, 64, BN);
  // bf16 outputs without read-modify-write go through the TMA-store epilogue
  args.tma_out = (splits == 1 && !out_f32 && !(args.epi & kEpiAccum)) ? 1 : 0;
  CUtensorMap mo = ma, mx = ma;  // placeholders when unused (never dereferenced)
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (args.tma_out) {
    mo = make_tma_2d_bf16(out.data_ptr(), N, M, out.stride(0), 64, 32);
    if (args.epi & kEpiGelu) mx = make_tma_2d_bf16(aux->data_ptr(), N, M, args.ldaux, 64, 32);
  } else if (args.red_out) {
    mo = make_tma_2d_f32(workspace->data_ptr(), N, M, N, 32, 32);
    C10_CUDA_CHECK(cudaMemsetAsync(workspace->data_ptr(), 0, static_cast<size_t>(M) * N * sizeof(float), stream));
  }
#define MNB_GEMM_CASE(BNV, AM, BMJ, ST)                                   \
  if (BN == BNV && a_mn == AM && b_mn == BMJ) {                            \
    launch_gemm<BNV, AM, BMJ, ST>(ma, mb, mo, mx, args, units, stream);    \
  } else
  const bool gelu_out = (args.epi & kEpiGelu) != 0;
  // TMA-store epilogues of K-major-A GEMMs can trade one pipeline stage for a
  // second staging box per epilogue warp (double-buffered stores): chosen by
  // MNB_GEMM_STAGES=3 (measured A/B switch; 4 stages by default).
  static const bool three_stage = [] {
    const char* e = std::getenv("MNB_GEMM_STAGES");
    return e != nullptr && std::string(e) == "3";
  }();
  if (gelu_out) {
    TORCH_CHECK(!a_mn && !b_mn, "the GELU epilogue is for the forward (K-major) layout");
    if (BN == 256) launch_gemm<256, false, false, 3>(ma, mb, mo, mx, args, units, stream);
    else launch_gemm<128, false, false, 3>(ma, mb, mo, mx, args, units, stream);
  } else if (three_stage && args.tma_out && !a_mn) {
    if (BN == 256 && !b_mn) launch_gemm<256, false, false, 3>(ma, mb, mo, mx, args, units, stream);
    else if (BN == 256) launch_gemm<256, false, true, 3>(ma, mb, mo, mx, args, units, stream);
    else if (!b_mn) launch_gemm<128, false, false, 3>(ma, mb, mo, mx, args, units, stream);
    else launch_gemm<128, false, true, 3>(ma, mb, mo, mx, args, units, stream);
  } else
  MNB_GEMM_CASE(256, false, false, 4)
  MNB_GEMM_CASE(256, false, true, 4)
  MNB_GEMM_CASE(256, true, false, 4)
  MNB_GEMM_CASE(256, true, true, 4)
  MNB_GEMM_CASE(128, false, false, 4)
  MNB_GEMM_CASE(128, false, true, 4)
  MNB_GEMM_CASE(128, true, false, 4)
  MNB_GEMM_CASE(128, true, true, 4) { TORCH_CHECK(false, "unsupported GEMM configuration"); }
#undef MNB_GEMM_CASE
  if (splits > 1) {
    const long long total4 = static_cast<long long>(M) * N / 4;
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<long long>((total4 + threads - 1) / threads, 148LL * 8));
    splitk_reduce_kernel<<<blocks, threads, 0, stream>>>(
        reinterpret_cast<const float*>(workspace->data_ptr()), 1,
        static_cast<long long>(M) * N, M, N, out.data_ptr(), out.stride(0), out_f32 ? 1 : 0,
        (epi & kEpiAccum) ? 1 : 0);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// Fused GEMM + collective (see the top of this file).  Called by the device
// communicator, which fills `ctx` for this call.
//   kFuseRS: a = X [M, K] (this rank's partial-sum input, all rows), b = W,
//            out = [M / world, N] (this rank's rows), bias [N] and resid
//            [M / world, N] are added once, after the reduction.
//   kFuseAG: a = X shard [M / world, K]; the gathered [M, K] is built in
//            this call's staging region (ctx.data[rank]); with rows % 128 == 0
//            the own rows are read in place from `a`, else the caller has
//            copied them into their block of the staging region.
//   *ag_base is the running total of increments of this mode's arrival
//   counters (advanced here by this launch's grid: one per CTA per rank).
void gemm_fused(int fuse, torch::Tensor a, torch::Tensor b, torch::Tensor out, bool b_mn,
                c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux,
                c10::optional<torch::Tensor> resid, int64_t epi, torch::Tensor status, const PeerCtx& ctx,
                uint32_t* ag_base, c10::optional<torch::Tensor> stamps) {
  c10::cuda::CUDAGuard guard(a.device());
  const int W = ctx.world;
  TORCH_CHECK(fuse == kFuseRS || fuse == kFuseAG, "unknown fused mode");
  TORCH_CHECK(ag_base != nullptr, "fused GEMMs need their arrival-counter base");
  const int64_t lda = row_stride(a, "A");
  const int64_t ldb = row_stride(b, "B");
  const int K = static_cast<int>(a.size(1));
  const int N = static_cast<int>(b_mn ? b.size(1) : b.size(0));
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "A and B disagree on K");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "N and K must be multiples of 8");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && (out.stride(0) % 8) == 0,
              "fused output must be bf16 with 16-byte rows");
  GemmArgs args{};
  args.N = N;
  args.K = K;
  args.status = status.data_ptr<int>();
  args.k_blocks_per_split = (K + kBK - 1) / kBK;
  args.splits = 1;
  args.out = out.data_ptr();
  args.ldo = out.stride(0);
  if (stamps) {
    TORCH_CHECK(stamps->scalar_type() == at::kLong && stamps->numel() >= 4 && stamps->is_cuda(), "stamps: int64 [4]");
    args.stamps = reinterpret_cast<unsigned long long*>(stamps->data_ptr());
  }
  CUtensorMap ma, mo, mx, mown;
  const bool wide = N >= 256;
  const int BN = wide ? 256 : 128;
  if (fuse == kFuseRS) {
    const int M = static_cast<int>(a.size(0));
    TORCH_CHECK(M % W == 0, "rows must divide evenly across ranks");
    TORCH_CHECK(out.size(0) == M / W && out.size(1) == N, "RS output must be [M / world, N]");
    TORCH_CHECK(lda == K, "A must be contiguous");
    args.M = M;
    args.rows_per_rank = M / W;
    if (bias) {
      TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "bias must be bf16 [N]");
      args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
    }
    if (resid) {
      TORCH_CHECK(resid->scalar_type() == at::kBFloat16 && resid->size(0) == M / W && resid->size(1) == N &&
                      resid->stride(1) == 1 && resid->stride(0) % 8 == 0,
                  "resid must be bf16 [M / world, N] with 16-byte rows");
      args.resid = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
      args.ldr = resid->stride(0);
    }
    args.epi = 0;
    args.tma_out = 0;
    ma = make_tma_2d_bf16(a.data_ptr(), K, M, lda, 64, kBM);
    mo = mx = mown = ma;
  } else {
    const int rows = static_cast<int>(a.size(0));
    const int M = rows * W;
    TORCH_CHECK(lda == K, "A shard must be contiguous");
    TORCH_CHECK(out.size(0) == M && out.size(1) == N, "AG output must be [M, N]");
    args.M = M;
    args.rows_per_rank = rows;
    args.ag_local = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
    args.epi = static_cast<int>(epi);
    if (bias) {
      TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "bias must be bf16 [N]");
      args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
      args.epi |= kEpiBias;
    }
    if (aux) {
      TORCH_CHECK(aux->scalar_type() == at::kBFloat16 && aux->stride(1) == 1, "aux must be bf16 row-major");
      args.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
      args.ldaux = aux->stride(0);
    }
    if (resid) {
      TORCH_CHECK(resid->scalar_type() == at::kBFloat16 && resid->stride(1) == 1, "resid must be bf16 row-major");
      args.resid = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
      args.ldr = resid->stride(0);
      args.epi |= kEpiResid;
    }
    TORCH_CHECK(!(args.epi & kEpiAccum), "AG-GEMM epilogues: bias, GELU, GELU', residual");
    TORCH_CHECK(!(args.epi & (kEpiGelu | kEpiGeluGrad)) || aux.has_value(), "GELU epilogues need aux");
    args.tma_out = 1;
    args.ag_own_map = rows % kBM == 0 ? 1 : 0;
    ma = make_tma_2d_bf16(ctx.data[ctx.rank], K, M, K, 64, kBM);
    mown = make_tma_2d_bf16(a.data_ptr(), K, rows, K, 64, kBM);
    mo = make_tma_2d_bf16(out.data_ptr(), N, M, out.stride(0), 64, 32);
    mx = (args.epi & kEpiGelu) ? make_tma_2d_bf16(aux->data_ptr(), N, M, args.ldaux, 64, 32) : mo;
  }
  CUtensorMap mb = b_mn ? make_tma_2d_bf16(b.data_ptr(), N, K, ldb, 64, 64)
                        : make_tma_2d_bf16(b.data_ptr(), K, N, ldb, 64, BN);
  const int units = ((args.M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  // one arrival per CTA of each rank on the matching counter row
  *ag_base += static_cast<uint32_t>(std::min(units, num_sms()));
  (fuse == kFuseAG ? args.ag_target : args.rs_target) = *ag_base;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const bool gelu = (args.epi & kEpiGelu) != 0;
#define MNB_FUSED(BNV, BMJ, ST, F)                                                   \
  if (BN == BNV && b_mn == BMJ) {                                                   \
    launch_gemm<BNV, false, BMJ, ST, F>(ma, mb, mo, mx, args, units, stream, ctx, &mown); \
    return;                                                                         \
  }
  if (fuse == kFuseRS) {
    MNB_FUSED(256, false, 4, kFuseRS)
    MNB_FUSED(256, true, 4, kFuseRS)
    MNB_FUSED(128, false, 4, kFuseRS)
    MNB_FUSED(128, true, 4, kFuseRS)
  } else if (gelu) {
    TORCH_CHECK(!b_mn, "the GELU epilogue is for the forward (K-major) layout");
    MNB_FUSED(256, false, 3, kFuseAG)
    MNB_FUSED(128, false, 3, kFuseAG)
  } else {
    MNB_FUSED(256, false, 4, kFuseAG)
    MNB_FUSED(256, true, 4, kFuseAG)
    MNB_FUSED(128, false, 4, kFuseAG)
    MNB_FUSED(128, true, 4, kFuseAG)
  }
#undef MNB_FUSED
  TORCH_CHECK(false, "unsupported fused GEMM configuration");
}


// FSDP: out [M, N] = x [M, K] @ B^T (+ bias), where B = rows [0, N) of a [N, K]
// weight at element offset w_off of a flattened parameter buffer that the
// ranks hold one shard each of (shards[p]: rank p's shard, `shard` elements).
// The launch also gathers the whole buffer into `flat` (kFuseAGW above).
// `counters`: uint32 [world * 16 + 1] of scratch (zeroed here).
void gemm_agw(torch::Tensor x, torch::Tensor flat, int64_t w_off, int64_t N, c10::optional<torch::Tensor> bias,
              torch::Tensor out, const std::vector<const void*>& shards, int64_t shard, torch::Tensor counters,
              torch::Tensor status, const PeerCtx& ctx, uint32_t* ag_base) {
  c10::cuda::CUDAGuard guard(x.device());
  const int W = ctx.world;
  TORCH_CHECK(static_cast<int>(shards.size()) == W, "one shard address per rank");
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && x.scalar_type() == at::kBFloat16, "x: contiguous bf16 [M, K]");
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1));
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0 && N > 0, "N and K must be multiples of 8");
  TORCH_CHECK(shard % 8 == 0 && shard > 0, "shards must be a positive multiple of 8 elements");
  TORCH_CHECK(flat.is_contiguous() && flat.scalar_type() == at::kBFloat16 && flat.numel() == shard * W,
              "flat: contiguous bf16 [world * shard]");
  TORCH_CHECK(w_off % 8 == 0 && w_off >= 0 && w_off + N * K <= shard * W, "the weight must lie in the buffer");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1 &&
                  out.stride(0) % 8 == 0,
              "out: bf16 [M, N] with 16-byte rows");
  TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= W * 16 + 1, "counters: int32 [world*16+1]");
  GemmArgs args{};
  args.M = M;
  args.N = static_cast<int>(N);
  args.K = K;
  args.status = status.data_ptr<int>();
  args.k_blocks_per_split = (K + kBK - 1) / kBK;
  args.splits = 1;
  args.out = out.data_ptr();
  args.ldo = out.stride(0);
  args.tma_out = 1;
  args.epi = 0;
  if (bias) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N && bias->is_contiguous(),
                "bias must be bf16 [N]");
    args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
    args.epi |= kEpiBias;
  }
  for (int p = 0; p < W; ++p) args.agw_src[p] = static_cast<const __nv_bfloat16*>(shards[p]);
  args.agw_flat = reinterpret_cast<__nv_bfloat16*>(flat.data_ptr());
  args.agw_shard = shard;
  const int64_t chunk = ((shard + 15) / 16 + 7) / 8 * 8;  // at most 16 chunks per shard
  args.agw_chunk = chunk;
  args.agw_nch = static_cast<int>((shard + chunk - 1) / chunk);
  args.agw_parts = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(64, chunk * 2 / 8192)));
  args.agw_w_off = w_off;
  args.agw_bias_off = -1;  // the bias is an ordinary tensor here
  auto chunk_of = [&](int64_t f) {
    const int64_t s = f / shard;
    return static_cast<int>(s * args.agw_nch + (f - s * shard) / chunk);
  };
  args.agw_pri_first = chunk_of(w_off);
  args.agw_pri_last = chunk_of(w_off + N * K - 1);
  args.agw_cnt = reinterpret_cast<uint32_t*>(counters.data_ptr());
  static const bool shallow = std::getenv("MNB_AGW_SHALLOW") != nullptr;  // A/B switch for benchmarks
  args.agw_shallow = shallow ? 1 : 0;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemsetAsync(counters.data_ptr(), 0, (W * args.agw_nch + 1) * sizeof(uint32_t), stream));
  const int BN = N >= 256 ? 256 : 128;
  CUtensorMap ma = make_tma_2d_bf16(x.data_ptr(), K, M, K, 64, kBM);
  CUtensorMap mb = make_tma_2d_bf16(args.agw_flat + w_off, K, static_cast<int>(N), K, 64, BN);
  CUtensorMap mo = make_tma_2d_bf16(out.data_ptr(), static_cast<int>(N), M, out.stride(0), 64, 32);
  const int units = ((M + kBM - 1) / kBM) * ((static_cast<int>(N) + BN - 1) / BN);
  // one start signal per CTA of each rank (the kCountRow counters it shares with kFuseAG)
  *ag_base += static_cast<uint32_t>(std::min(units, num_sms()));
  args.ag_target = *ag_base;
  if (BN == 256) launch_gemm<256, false, false, 4, kFuseAGW>(ma, mb, mo, mo, args, units, stream, ctx, &ma);
  else launch_gemm<128, false, false, 4, kFuseAGW>(ma, mb, mo, mo, args, units, stream, ctx, &ma);
}

}  // namespace mnb
