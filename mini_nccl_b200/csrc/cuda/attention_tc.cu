// Causal flash-attention forward on the 5th-generation tensor cores (tcgen05).
//
// One CTA computes 128 query rows of one (batch, head).  Roles:
//   warp 0      TMA producer: Q once, then K_j / V_j tiles (128 keys x D,
//               128-byte swizzle) into a KV_STAGES-deep ring.
//   warp 1      TMEM owner; one lane issues the MMAs:
//                 S_j  = Q K_j^T        (M=128, N=128 keys, K=D)   -> TMEM cols [0, 128)
//                 O_j  = P_j V_j        (M=128, N=D,   K=128 keys) -> TMEM cols [128, 128+D)
//               P_j comes from shared memory (bf16, K-major); V_j is read
//               MN-major straight from its TMA tile.
//   warps 2..5  softmax: thread = one query row.  tcgen05.ld S_j, online
//               softmax in base 2, write P_j to shared memory, then fold
//               O_{j-1} from TMEM into a register accumulator with the
//               running rescale; finally normalise and store O and the LSE.
// S_{j+1} = Q K_{j+1}^T is issued as soon as the softmax has read S_j, so the
// tensor core overlaps the softmax of the previous tile.  256 TMEM columns
// per CTA lets two CTAs share an SM.  All waits are bounded (status word).
//
// Same algorithm as the mma.sync kernel in attention.cu (FlashAttention-2
// online softmax, causal tile skipping); inputs/outputs identical.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "common.cuh"

namespace mnb {

CUtensorMap make_tma_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                             uint32_t box_inner, uint32_t box_outer);
CUtensorMap make_tma_2d_f32(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                            uint32_t box_inner, uint32_t box_outer);

namespace fatc {

constexpr int kQ = 128;        // queries per CTA
constexpr int kKV = 128;       // keys per tile
constexpr int kSoftWarps = 8;  // two per TMEM lane quadrant, each owning half the keys
constexpr int kSoftThreads = 32 * kSoftWarps;
constexpr int kThreads = 64 + kSoftThreads;  // producer, MMA, softmax warps
constexpr float kLog2e = 1.4426950408889634f;

MNB_DEVICE void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
MNB_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for x <= 0 on the FMA and integer pipes, to take part of the
// softmax's exponentials off the MUFU unit (the forward's bottleneck).
// x = n + f with n = round(x) (adding and subtracting 1.5 * 2^23 rounds to
// the nearest integer in plain float adds; the integer is read off the sum's
// low mantissa bits) and f in [-1/2, 1/2]; 2^f from the cubic
// 1 + c1 f + c2 f^2 + c3 f^3 with c1..c3 an iteratively reweighted least-
// squares fit of 2^f on [-1/2, 1/2] for relative error (computed for this
// library: maximum relative error 1.0e-4, under bf16's half-ulp of 2^-9);
// 2^n by adding n to the exponent field.  Inputs below -126 give about
// 2^-126 (the probabilities are rounded to bf16 next).
MNB_DEVICE float exp2_poly(float x) {
  constexpr float c1 = 0.6932827186256372f, c2 = 0.2422078019971109f, c3 = 0.055007628266016344f;
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x = fmaxf(x, -126.f);
  const float t = x + kRound;
  const int n = __float_as_int(t) - 0x4B400000;
  const float f = x - (t - kRound);
  const float p = fmaf(fmaf(fmaf(c3, f, c2), f, c1), f, 1.0f);
  return __int_as_float(__float_as_int(p) + (n << 23));
}

MNB_DEVICE void softmax_barrier() { asm volatile("bar.sync 1, %0;" ::"n"(kSoftThreads) : "memory"); }

template <int D, int KV_STAGES>
struct Smem {
  static constexpr uint32_t q_bytes = kQ * D * 2;
  static constexpr uint32_t kv_bytes = kKV * D * 2;
  static constexpr uint32_t p_bytes = kQ * kKV * 2;
  static constexpr uint32_t q_off = 0;
  static constexpr uint32_t k_off = q_bytes;
  static constexpr uint32_t v_off = k_off + KV_STAGES * kv_bytes;
  static constexpr uint32_t p_off = v_off + KV_STAGES * kv_bytes;
  // float [3][2][kQ]: row-max exchange for even / odd tiles, then the row sums
  static constexpr uint32_t red_off = p_off + p_bytes;
  static constexpr uint32_t bar_off = red_off + 3 * 2 * kQ * 4;
  static constexpr int n_bars = 7 + 4 * KV_STAGES;
  static constexpr uint32_t total = bar_off + n_bars * 8 + 16 + 1024;
};

template <int D, int KV_STAGES>
__global__ void __launch_bounds__(kThreads, D == 64 ? 2 : 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_qkv, __nv_bfloat16* __restrict__ o,
                     float* __restrict__ lse, int H, int T, float scale, int* status) {
  using S = Smem<D, KV_STAGES>;
  constexpr uint32_t kTmemCols = 256;
  constexpr uint32_t kIdescS = idesc_bf16(kQ, kKV, false, false);
  constexpr uint32_t kIdescO = idesc_bf16(kQ, D, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::bar_off);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::n_bars);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0, s_full = b0 + 8, s_free = b0 + 16, p_full = b0 + 24, p_free = b0 + 32,
                 o_full = b0 + 40, o_free = b0 + 48;
  // K_j is released as soon as S_j has been computed, V_j once P_j V_j has:
  // separate barriers so a single-stage ring cannot deadlock on V.
  const uint32_t k_full0 = b0 + 56, v_full0 = k_full0 + 8 * KV_STAGES, k_empty0 = v_full0 + 8 * KV_STAGES,
                 v_empty0 = k_empty0 + 8 * KV_STAGES;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // grid (B*H, query tiles), x fastest: every head's longest causal rows are
  // launched before any head's shorter ones (longest work first over the whole grid)
  const int qt = gridDim.y - 1 - blockIdx.y;
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int q0 = qt * kQ;
  const int C = H * D;
  const int n_kv = min(qt + 1, (T + kKV - 1) / kKV);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, kSoftThreads);
    mbar_init(p_full, kSoftThreads);
    mbar_init(p_free, 1);
    mbar_init(o_full, 1);
    mbar_init(o_free, kSoftThreads);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(k_full0 + 8 * s, 1);
      mbar_init(v_full0 + 8 * s, 1);
      mbar_init(k_empty0 + 8 * s, 1);
      mbar_init(v_empty0 + 8 * s, 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&map_qkv);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + kKV;

  if (warp == 0) {
    if (lane == 0) {
      const int row0 = b * T;
      mbar_arrive_expect_tx(q_full, S::q_bytes);
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        tma_load_2d(sbase + S::q_off + c * (kQ * 128), &map_qkv, h * D + c * 64, row0 + q0, q_full);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        if (!mbar_wait(k_empty0 + 8 * st, ph ^ 1, status)) break;
        mbar_arrive_expect_tx(k_full0 + 8 * st, S::kv_bytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(sbase + S::k_off + st * S::kv_bytes + c * (kKV * 128), &map_qkv, C + h * D + c * 64,
                      row0 + j * kKV, k_full0 + 8 * st);
        if (!mbar_wait(v_empty0 + 8 * st, ph ^ 1, status)) break;
        mbar_arrive_expect_tx(v_full0 + 8 * st, S::kv_bytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(sbase + S::v_off + st * S::kv_bytes + c * (kKV * 128), &map_qkv, 2 * C + h * D + c * 64,
                      row0 + j * kKV, v_full0 + 8 * st);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, status);
      auto pv = [&](int i) -> bool {
        const int st = i % KV_STAGES;
        if (!mbar_wait(v_full0 + 8 * st, (i / KV_STAGES) & 1, status)) return false;
        if (!mbar_wait(p_full, i & 1, status)) return false;
        if (!mbar_wait(o_free, (i & 1) ^ 1, status)) return false;
        tc_fence_after();
        const uint32_t pa = sbase + S::p_off;
        const uint32_t vb = sbase + S::v_off + st * S::kv_bytes;
#pragma unroll
        for (int kk = 0; kk < kKV / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(pa + (kk / 4) * (kQ * 128) + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(vb + kk * 2048, kKV * 128, 1024);
          tc_mma(tO, ad, bd, kIdescO, kk > 0 ? 1u : 0u);
        }
        tc_commit(o_full);
        tc_commit(p_free);
        tc_commit(v_empty0 + 8 * st);
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % KV_STAGES;
        ok = mbar_wait(k_full0 + 8 * st, (j / KV_STAGES) & 1, status) && mbar_wait(s_free, (j & 1) ^ 1, status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t qa = sbase + S::q_off;
        const uint32_t kb = sbase + S::k_off + st * S::kv_bytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(qa + (kk / 4) * (kQ * 128) + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(kb + (kk / 4) * (kKV * 128) + (kk % 4) * 32, 16, 1024);
          tc_mma(tS, ad, bd, kIdescS, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        tc_commit(k_empty0 + 8 * st);
        if (j >= 1) ok = pv(j - 1);
      }
      if (ok && n_kv > 0) pv(n_kv - 1);
    }
  } else {
    // softmax: warp w owns TMEM lanes 32*(w%4) (query rows); warps w and w+4
    // split each row's 128 keys (and the D output columns) in halves.
    const int qd = warp & 3;
    const int half = (warp - 2) / 4;
    const int r = qd * 32 + lane;  // row within the tile
    const int qrow = q0 + r;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_cols = tS + lane_base + half * (kKV / 2);
    const uint32_t o_cols = tO + lane_base + half * (D / 2);
    float* red = reinterpret_cast<float*>(sm + S::red_off);  // [tile parity][half][row]
    const float sl2 = scale * kLog2e;
    float oacc[D / 2];
#pragma unroll
    for (int i = 0; i < D / 2; ++i) oacc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;  // m_run in scaled log2 units
    bool ok = true;
    uint8_t* pbase = sm + S::p_off + half * (kQ * 128);      // this half's 64-key atom
    for (int j = 0; j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, status));
      if (!ok) break;
      tc_fence_after();
      const int k0 = j * kKV + half * (kKV / 2);
      const bool masked = (j * kKV + kKV - 1 > q0) || (j * kKV + kKV > T);
      // pass 1: this half-row's max of the raw scores
      float mraw = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kKV / 64; ++c) {
        float sv[32];
        tmem_ld_32(s_cols + c * 32, sv);
        if (masked) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = k0 + c * 32 + i;
            if (key <= qrow && key < T) mraw = fmaxf(mraw, sv[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) mraw = fmaxf(mraw, sv[i]);
        }
      }
      red[(j & 1) * 2 * kQ + half * kQ + r] = mraw;
      softmax_barrier();
      mraw = fmaxf(mraw, red[(j & 1) * 2 * kQ + (half ^ 1) * kQ + r]);
      const float mx = fmaxf(m_run, mraw * sl2);
      const float alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - mx);
      m_run = mx;
      if (j >= 1) {
        ok = __all_sync(0xffffffffu, mbar_wait(p_free, (j - 1) & 1, status));
        if (!ok) break;
      }
      // pass 2: p = 2^(s*scale*log2e - m), row sum, bf16 P into this half's atom
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < kKV / 64; ++c) {
        float sv[32];
        tmem_ld_32(s_cols + c * 32, sv);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float pv = fast_exp2(fmaf(sv[i], sl2, -mx));
          if (masked) {
            const int key = k0 + c * 32 + i;
            pv = (key <= qrow && key < T) ? pv : 0.f;
          }
          sv[i] = pv;
          rs += pv;
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int chunk = c * 4 + q8;  // 16-byte chunk within the 64-key atom
          const uint32_t off = (r / 8) * 1024 + (r % 8) * 128 + ((chunk ^ (r % 8)) * 16);
          const float* f = sv + 8 * q8;
          *reinterpret_cast<uint4*>(pbase + off) =
              make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                         pack_bf16x2(f[6], f[7]));
        }
      }
      tc_fence_before();
      mbar_arrive(s_free);
      l_run = l_run * alpha + rs;
      fence_async_smem();
      mbar_arrive(p_full);
      if (j >= 1) {
        ok = __all_sync(0xffffffffu, mbar_wait(o_full, (j - 1) & 1, status));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          float ov[32];
          tmem_ld_32(o_cols + c * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) oacc[c * 32 + i] = fmaf(oacc[c * 32 + i], alpha_prev, ov[i]);
        }
        tc_fence_before();
        mbar_arrive(o_free);
      }
      alpha_prev = alpha;
    }
    if (ok && n_kv > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(o_full, (n_kv - 1) & 1, status));
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          float ov[32];
          tmem_ld_32(o_cols + c * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) oacc[c * 32 + i] = fmaf(oacc[c * 32 + i], alpha_prev, ov[i]);
        }
        tc_fence_before();
      }
    }
    // the two halves' row sums share m_run, so the full sum is their total
    red[4 * kQ + half * kQ + r] = l_run;
    softmax_barrier();
    const float l_tot = l_run + red[4 * kQ + (half ^ 1) * kQ + r];
    if (ok && qrow < T) {
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      __nv_bfloat16* orow = o + (static_cast<long long>(b) * T + qrow) * C + h * D + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint4 v = make_uint4(pack_bf16x2(oacc[8 * c] * inv, oacc[8 * c + 1] * inv),
                             pack_bf16x2(oacc[8 * c + 2] * inv, oacc[8 * c + 3] * inv),
                             pack_bf16x2(oacc[8 * c + 4] * inv, oacc[8 * c + 5] * inv),
                             pack_bf16x2(oacc[8 * c + 6] * inv, oacc[8 * c + 7] * inv));
        *reinterpret_cast<uint4*>(orow + 8 * c) = v;
      }
      if (half == 0) lse[(static_cast<long long>(b) * H + h) * T + qrow] = (m_run + log2f(l_tot)) / kLog2e;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ===========================================================================
// Backward on tcgen05.  One CTA owns 128 keys (tile j) of one (batch, head)
// and walks the query tiles i >= j (causal).  TMEM lanes are keys:
//   S^T  = K_j Q_i^T          (M=128 keys, N=128 queries, K=D)  cols [0, 128)
//   dP^T = V_j dO_i^T         (same shape)                      cols [128, 256)
//   dV  += P^T dO_i           (M=keys, N=D, K=queries)          cols [256, 256+D)
//   dK  += dS^T Q_i           (M=keys, N=D, K=queries)          cols [256+D, 256+2D)
//   dQ_i = dS K_j             (M=queries, N=D, K=keys)          cols [128, 128+D) (reuses dP^T)
// The compute warps turn S^T into P^T = exp(S^T*scale - lse) and dP^T into
// dS^T = scale * P^T (dP^T - delta), both bf16 in 128-byte-swizzled shared
// memory.  The same dS^T tile is the K-major A operand of dK and, read
// MN-major (queries contiguous), the A operand of dQ.  dQ_i leaves TMEM
// through a 128-byte-swizzled fp32 staging box in shared memory and is added
// into a [B, T, C] fp32 accumulator by TMA reduce-add (the adds run at L2, the
// compute warps do not wait for them); dK and dV are written once at the end.
// For D = 64 dQ has its own TMEM columns, so dP^T of the next query tile does
// not wait for dQ to be read out.  Warp roles: producer, MMA, then PARTS x 4
// compute warps; compute warp w serves TMEM lanes 32 (w % 4) .. +31 and the
// column part (w - 2) / 4 of every tile it reads (S^T, dP^T: 128 / PARTS
// columns; dQ, dK, dV: D / PARTS).  PARTS = 4 puts four warps on each
// scheduler to hide the TMEM, shared-memory and MUFU latencies of the
// exponentials and dS; PARTS = 2 needs fewer registers per thread.
// ===========================================================================
constexpr int bwd_threads(int parts) { return 64 + 128 * parts; }

template <int D, int STAGES>
struct BwdSmem {
  static constexpr uint32_t tile = 128 * D * 2;  // one [128 rows x D] bf16 tile
  static constexpr uint32_t k_off = 0;
  static constexpr uint32_t v_off = tile;
  static constexpr uint32_t stage_bytes = 2 * tile + 2 * 128 * 4;  // Q, dO, lse, delta
  static constexpr uint32_t st_off = 2 * tile;
  static constexpr uint32_t p_off = st_off + STAGES * stage_bytes;
  static constexpr uint32_t ds_off = p_off + 128 * 128 * 2;
  static constexpr uint32_t dq_off = ds_off + 128 * 128 * 2;  // two [128 x 32] fp32 staging boxes
  static constexpr uint32_t bar_off = dq_off + 2 * 128 * 128;
  static constexpr int n_bars = 16 + 2 * STAGES;
  static constexpr uint32_t total = bar_off + n_bars * 8 + 16 + 1024;
  static_assert(st_off % 1024 == 0 && p_off % 1024 == 0 && ds_off % 1024 == 0 && dq_off % 1024 == 0,
                "1 KiB aligned tiles");
  static_assert(total <= 232448, "shared memory per CTA");
};

MNB_DEVICE float2 ld_shared_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
MNB_DEVICE void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// Swizzled row addressing shared by the stores below: row `r` of a [128 x 128 B]
// atom starts at row_base(r); its 16-byte chunk k sits at slot k ^ (r % 8).
MNB_DEVICE uint32_t row_base(uint32_t atom, int r) { return atom + (r / 8) * 1024 + (r % 8) * 128; }

// 16 packed bf16 pairs (32 values) -> chunk group c (chunks 4c..4c+3) of a swizzled bf16 row.
MNB_DEVICE void store_row_words(uint32_t rowb, int x, int c, const uint32_t* w) {
#pragma unroll
  for (int q8 = 0; q8 < 4; ++q8)
    st_shared_v4(rowb + (((c * 4 + q8) ^ x) << 4), w[4 * q8], w[4 * q8 + 1], w[4 * q8 + 2], w[4 * q8 + 3]);
}
// 32 floats -> chunk group c of a swizzled bf16 row.
MNB_DEVICE void store_row_bf16(uint32_t rowb, int x, int c, const float* v) {
#pragma unroll
  for (int q8 = 0; q8 < 4; ++q8) {
    const float* f = v + 8 * q8;
    st_shared_v4(rowb + (((c * 4 + q8) ^ x) << 4), pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                 pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
}
// 32 floats -> one swizzled fp32 row (128 bytes, 8 chunks).
MNB_DEVICE void store_row_f32(uint32_t rowb, int x, const float* v) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    st_shared_v4(rowb + ((k ^ x) << 4), __float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                 __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
}

// ===========================================================================
// Forward, two query tiles per CTA (head dim 64, T % 256 == 0).
//
// The CTA owns query tiles A = [q0, q0+128) and B = [q0+128, q0+256) of one
// (batch, head); each has its own S (TMEM cols [0,128) / [128,256)), O
// accumulator ([256,320) / [320,384)) and P tile in shared memory, and its own
// softmax warpgroup (warps 2-5 for A, 6-9 for B) in which every thread owns
// one full query row, so the row max and sum need no exchange between warps.
// The MMA warp issues S_A(j), PV_A(j-1), S_B(j), PV_B(j-1): while one
// warpgroup runs the exponentials of its tile the tensor core works on the
// other tile's products.  K_j / V_j are loaded once for both tiles.  Same
// online softmax, outputs and LSE as fa_fwd_tc_kernel.
// ===========================================================================
constexpr int kPPThreads = 64 + 256;

struct PPSmem {
  static constexpr uint32_t tile = 128 * 64 * 2;  // [128 rows x 64] bf16: one 128-byte-swizzle atom
  static constexpr uint32_t q_off = 0;            // Q_A, Q_B
  static constexpr uint32_t k_off = 2 * tile;     // two stages
  static constexpr uint32_t v_off = 4 * tile;     // two stages
  static constexpr uint32_t p_off = 6 * tile;     // P_A, P_B: [128 x 128 keys] bf16, two atoms each
  static constexpr uint32_t bar_off = 10 * tile;
  static constexpr int n_bars = 1 + 12 + 8;
  static constexpr uint32_t total = bar_off + n_bars * 8 + 16 + 1024;
};

// kPoly: half of the softmax's exponentials as exp2_poly on the FMA pipe
// (true), or all of them on MUFU (false).  kPacked: the row max with
// three-input max and the scaling, row sums and O rescaling in f32x2 pairs
// (fewer instructions, same rounding; measured no faster), or all scalar.
template <bool kPoly, bool kPacked>
__global__ void __launch_bounds__(kPPThreads, 1)
    fa_fwd_pp_kernel(const __grid_constant__ CUtensorMap map_qkv, __nv_bfloat16* __restrict__ o,
                     float* __restrict__ lse, int H, int T, float scale, int* status) {
  using S = PPSmem;
  constexpr int D = 64;
  constexpr uint32_t kIdescS = idesc_bf16(128, 128, false, false);
  constexpr uint32_t kIdescO = idesc_bf16(128, D, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::bar_off);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::n_bars);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0;
  // per tile t: s_full, s_free, p_full, p_free, o_full, o_free
  auto tb = [&](int k, int t) { return b0 + 8 * (1 + 2 * k + t); };
  const uint32_t kv0 = b0 + 8 * 13;  // k_full[2], k_empty[2], v_full[2], v_empty[2]
  auto k_full = [&](int st) { return kv0 + 8 * st; };
  auto k_empty = [&](int st) { return kv0 + 16 + 8 * st; };
  auto v_full = [&](int st) { return kv0 + 32 + 8 * st; };
  auto v_empty = [&](int st) { return kv0 + 48 + 8 * st; };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int pair = gridDim.y - 1 - blockIdx.y;  // longest causal rows of every head first
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int q0 = pair * 256;
  const int C = H * D;
  const int n_b = 2 * pair + 2;  // key tiles of tile B; tile A has one fewer

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(tb(0, t), 1);    // s_full
      mbar_init(tb(1, t), 128);  // s_free
      mbar_init(tb(2, t), 128);  // p_full
      mbar_init(tb(3, t), 1);    // p_free
      mbar_init(tb(4, t), 1);    // o_full
      mbar_init(tb(5, t), 128);  // o_free
    }
    for (int st = 0; st < 2; ++st) {
      mbar_init(k_full(st), 1);
      mbar_init(k_empty(st), 1);
      mbar_init(v_full(st), 1);
      mbar_init(v_empty(st), 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&map_qkv);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const int row0 = b * T;
      mbar_arrive_expect_tx(q_full, 2 * S::tile);
      tma_load_2d(sbase + S::q_off, &map_qkv, h * D, row0 + q0, q_full);
      tma_load_2d(sbase + S::q_off + S::tile, &map_qkv, h * D, row0 + q0 + 128, q_full);
      for (int j = 0; j < n_b; ++j) {
        const int st = j % 2;
        const uint32_t ph = (j / 2) & 1;
        if (!mbar_wait(k_empty(st), ph ^ 1, status)) break;
        mbar_arrive_expect_tx(k_full(st), S::tile);
        tma_load_2d(sbase + S::k_off + st * S::tile, &map_qkv, C + h * D, row0 + j * 128, k_full(st));
        if (!mbar_wait(v_empty(st), ph ^ 1, status)) break;
        mbar_arrive_expect_tx(v_full(st), S::tile);
        tma_load_2d(sbase + S::v_off + st * S::tile, &map_qkv, 2 * C + h * D, row0 + j * 128, v_full(st));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, status);
      auto mma_s = [&](int t, int j) -> bool {  // S_t = Q_t K_j^T
        if (!mbar_wait(tb(1, t), (j & 1) ^ 1, status)) return false;
        tc_fence_after();
        const uint32_t qa = sbase + S::q_off + t * S::tile, kb = sbase + S::k_off + (j % 2) * S::tile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma(tmem + 128 * t, smem_desc_sw128(qa + kk * 32, 16, 1024), smem_desc_sw128(kb + kk * 32, 16, 1024),
                 kIdescS, kk > 0 ? 1u : 0u);
        tc_commit(tb(0, t));
        return true;
      };
      auto mma_pv = [&](int t, int j) -> bool {  // O_t = P_t V_j
        if (!mbar_wait(tb(2, t), j & 1, status) || !mbar_wait(tb(5, t), (j & 1) ^ 1, status)) return false;
        tc_fence_after();
        const uint32_t pa = sbase + S::p_off + t * 2 * S::tile, vb = sbase + S::v_off + (j % 2) * S::tile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma(tmem + 256 + D * t, smem_desc_sw128(pa + (kk / 4) * S::tile + (kk % 4) * 32, 16, 1024),
                 smem_desc_sw128(vb + kk * 2048, S::tile, 1024), kIdescO, kk > 0 ? 1u : 0u);
        tc_commit(tb(4, t));
        tc_commit(tb(3, t));
        return true;
      };
#pragma unroll 1
      for (int j = 0; j <= n_b && ok; ++j) {
        if (j < n_b) {
          if (!(ok = mbar_wait(k_full(j % 2), (j / 2) & 1, status))) break;
          tc_fence_after();
        }
        if (j >= 1) {
          if (!(ok = mbar_wait(v_full((j - 1) % 2), ((j - 1) / 2) & 1, status))) break;
          tc_fence_after();
        }
        for (int t = 0; t < 2 && ok; ++t) {
          const int n_t = n_b - 1 + t;
          if (j < n_t) ok = mma_s(t, j);
          if (ok && j >= 1 && j <= n_t) ok = mma_pv(t, j - 1);
        }
        if (!ok) break;
        if (j < n_b) tc_commit(k_empty(j % 2));
        if (j >= 1) tc_commit(v_empty((j - 1) % 2));
      }
    }
  } else {
    const int t = (warp - 2) / 4;  // query tile of this warpgroup
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int qrow = q0 + t * 128 + r;
    const int n = n_b - 1 + t;
    const int diag = n - 1;  // the one key tile that needs the causal mask
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_cols = tmem + 128 * t + lane_base, o_cols = tmem + 256 + D * t + lane_base;
    const uint32_t s_full = tb(0, t), s_free = tb(1, t), p_full = tb(2, t), p_free = tb(3, t), o_full = tb(4, t),
                   o_free = tb(5, t);
    const int x = r % 8;
    const uint32_t p_row = row_base(sbase + S::p_off + t * 2 * S::tile, r);
    const float sl2 = scale * kLog2e;
    float oacc[D];
#pragma unroll
    for (int i = 0; i < D; ++i) oacc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;  // m_run in scaled log2 units
    auto fold = [&](int j) -> bool {  // oacc = oacc * alpha_prev + O(j)
      if (!__all_sync(0xffffffffu, mbar_wait(o_full, j & 1, status))) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float ov[32];
        tmem_ld_32(o_cols + c * 32, ov);
        if constexpr (kPacked) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 r = fma2(make_float2(oacc[c * 32 + i], oacc[c * 32 + i + 1]), splat2(alpha_prev),
                                  make_float2(ov[i], ov[i + 1]));
            oacc[c * 32 + i] = r.x;
            oacc[c * 32 + i + 1] = r.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) oacc[c * 32 + i] = fmaf(oacc[c * 32 + i], alpha_prev, ov[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(o_free);
      return true;
    };
    bool ok = true;
#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, status)))) break;
      tc_fence_after();
      const bool masked = j == diag;
      const int k0 = j * 128;
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float sv[32];
        tmem_ld_32(s_cols + c * 32, sv);
        if (masked) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (k0 + c * 32 + i <= qrow) mx = fmaxf(mx, sv[i]);
        } else if constexpr (kPacked) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) mx = max3f(mx, sv[i], sv[i + 1]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, sv[i]);
        }
      }
      const float m_new = fmaxf(m_run, mx * sl2);
      const float alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_new);
      if (j >= 1 && !(ok = __all_sync(0xffffffffu, mbar_wait(p_free, (j - 1) & 1, status)))) break;
      float rs = 0.f;
      float2 rs2 = make_float2(0.f, 0.f);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float sv[32];
        tmem_ld_32(s_cols + c * 32, sv);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float x0, x1;
          if constexpr (kPacked) {
            const float2 xs = fma2(make_float2(sv[i], sv[i + 1]), splat2(sl2), splat2(-m_new));
            x0 = xs.x;
            x1 = xs.y;
          } else {
            x0 = fmaf(sv[i], sl2, -m_new);
            x1 = fmaf(sv[i + 1], sl2, -m_new);
          }
          // with kPoly, every second exponential as a polynomial on the FMA pipe
          float p0 = fast_exp2(x0);
          float p1 = kPoly ? exp2_poly(x1) : fast_exp2(x1);
          if (masked) {
            if (k0 + c * 32 + i > qrow) p0 = 0.f;
            if (k0 + c * 32 + i + 1 > qrow) p1 = 0.f;
          }
          if constexpr (kPacked) {
            rs2 = add2(rs2, make_float2(p0, p1));
          } else {
            rs += p0 + p1;
          }
          w[i / 2] = pack_bf16x2(p0, p1);
        }
        store_row_words(p_row + (c / 2) * S::tile, x, c % 2, w);
      }
      tc_fence_before();
      mbar_arrive(s_free);
      fence_async_smem();
      mbar_arrive(p_full);
      if constexpr (kPacked) rs = rs2.x + rs2.y;
      l_run = l_run * alpha + rs;
      if (j >= 1 && !(ok = fold(j - 1))) break;
      alpha_prev = alpha;
      m_run = m_new;
    }
    if (ok) ok = fold(n - 1);
    if (ok) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = o + (static_cast<long long>(b) * T + qrow) * C + h * D;
#pragma unroll
      for (int c = 0; c < D / 8; ++c)
        *reinterpret_cast<uint4*>(orow + 8 * c) =
            make_uint4(pack_bf16x2(oacc[8 * c] * inv, oacc[8 * c + 1] * inv),
                       pack_bf16x2(oacc[8 * c + 2] * inv, oacc[8 * c + 3] * inv),
                       pack_bf16x2(oacc[8 * c + 4] * inv, oacc[8 * c + 5] * inv),
                       pack_bf16x2(oacc[8 * c + 6] * inv, oacc[8 * c + 7] * inv));
      lse[(static_cast<long long>(b) * H + h) * T + qrow] = (m_run + log2f(l_run)) / kLog2e;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, int STAGES, int PARTS>
__global__ void __launch_bounds__(bwd_threads(PARTS), 1)
    fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap map_qkv, const __grid_constant__ CUtensorMap map_do,
                     const __grid_constant__ CUtensorMap map_dq, const float* __restrict__ lse,
                     const float* __restrict__ delta, __nv_bfloat16* __restrict__ dqkv, int H, int T, float scale,
                     int* status) {
  using S = BwdSmem<D, STAGES>;
  constexpr uint32_t kTmemCols = 512;
  constexpr bool kOwnDq = 128 + 128 + 3 * D <= 512;  // dQ in its own columns (D = 64)
  constexpr bool kAhead = kOwnDq && STAGES >= 2;      // next tile's S issued before this tile's dK / dQ
  constexpr int kCompute = 128 * PARTS;                // compute threads
  constexpr int kSCols = 128 / PARTS;                  // S^T / dP^T columns of one part
  constexpr int kDCols = D / PARTS;                    // dQ / dK / dV columns of one part
  constexpr int kFill = kDCols < 32 ? kDCols : 32;     // dQ columns per staging-box fill
  constexpr int kPerBox = 32 / kFill;                  // parts sharing one [128 x 32] fp32 box
  static_assert(PARTS == 2 || PARTS == 4, "two or four column parts");
  static_assert(kSCols % 32 == 0 && kDCols % 16 == 0, "whole TMEM loads");
  static_assert(PARTS / kPerBox == 2, "two dQ staging boxes");
  constexpr uint32_t kIdSq = idesc_bf16(128, 128, false, false);  // S^T, dP^T
  constexpr uint32_t kIdKV = idesc_bf16(128, D, false, true);     // dV, dK
  constexpr uint32_t kIdQ = idesc_bf16(128, D, true, true);       // dQ
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::bar_off);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::n_bars);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t kv_full = b0, s_full = b0 + 8, s_free = b0 + 16, dp_full = b0 + 24, p_full = b0 + 32,
                 p_free = b0 + 40, ds_full = b0 + 48, ds_free = b0 + 56, dq_full = b0 + 64, dq_free = b0 + 72,
                 acc_full = b0 + 80;
  const uint32_t q_full0 = b0 + 96, q_empty0 = q_full0 + 8 * STAGES;
  const uint32_t stg_free0 = q_empty0 + 8 * STAGES, stg_full0 = stg_free0 + 16;  // [2] each, one per dQ staging box

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // grid (B*H, key tiles), x fastest: the key tiles with the most query tiles
  // (j = 0) of every head are launched first
  const int j = blockIdx.y;
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int C = H * D;
  const int n_q = T / 128;
  const int n_it = n_q - j;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, kCompute);
    mbar_init(dp_full, 1);
    mbar_init(p_full, kCompute);
    mbar_init(p_free, 1);
    mbar_init(ds_full, kCompute);
    mbar_init(ds_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kCompute);
    mbar_init(acc_full, 1);
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(q_full0 + 8 * st, 1);
      mbar_init(q_empty0 + 8 * st, 1);
    }
    for (int hf = 0; hf < 2; ++hf) {
      mbar_init(stg_free0 + 8 * hf, 1);
      mbar_init(stg_full0 + 8 * hf, 128 * kPerBox);
    }
    fence_mbar_init();
    tma_prefetch_desc(&map_qkv);
    tma_prefetch_desc(&map_do);
    tma_prefetch_desc(&map_dq);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tP = tmem + 128, tV = tmem + 256, tK = tmem + 256 + D;
  const uint32_t tQ = kOwnDq ? tmem + 256 + 2 * D : tP;

  if (warp == 0) {
    if (lane == 0) {
      const int row0 = b * T;
      mbar_arrive_expect_tx(kv_full, 2 * S::tile);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sbase + S::k_off + c * 16384, &map_qkv, C + h * D + c * 64, row0 + j * 128, kv_full);
        tma_load_2d(sbase + S::v_off + c * 16384, &map_qkv, 2 * C + h * D + c * 64, row0 + j * 128, kv_full);
      }
#pragma unroll 1
      for (int it = 0; it < n_it; ++it) {
        const int i = j + it, st = it % STAGES;
        if (!mbar_wait(q_empty0 + 8 * st, ((it / STAGES) & 1) ^ 1, status)) break;
        const uint32_t qf = q_full0 + 8 * st;
        const uint32_t so = sbase + S::st_off + st * S::stage_bytes;
        mbar_arrive_expect_tx(qf, 2 * S::tile + 2 * 128 * 4);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(so + c * 16384, &map_qkv, h * D + c * 64, row0 + i * 128, qf);
          tma_load_2d(so + S::tile + c * 16384, &map_do, h * D + c * 64, row0 + i * 128, qf);
        }
        const float* lsrc = lse + (static_cast<long long>(b) * H + h) * T + i * 128;
        const float* dsrc = delta + (static_cast<long long>(b) * H + h) * T + i * 128;
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], 512, [%2];"
                     ::"r"(so + 2 * S::tile), "l"(lsrc), "r"(qf) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], 512, [%2];"
                     ::"r"(so + 2 * S::tile + 512), "l"(dsrc), "r"(qf) : "memory");
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(kv_full, 0, status);
      const uint32_t ka0 = sbase + S::k_off, va0 = sbase + S::v_off;
      const uint32_t pa0 = sbase + S::p_off, dsa0 = sbase + S::ds_off;
      // Shared-memory operand addresses of query tile `it`, opaque to the
      // compiler so the ~40 descriptors are rebuilt per tile instead of being
      // hoisted into registers (and from there into local memory).
      struct Ops { uint32_t ka, va, pa, dsa, qa, doa; };
      auto ops = [&](int it) {
        Ops o{ka0, va0, pa0, dsa0, sbase + S::st_off + (it % STAGES) * S::stage_bytes, 0};
        o.doa = o.qa + S::tile;
        asm volatile("" : "+r"(o.ka), "+r"(o.va), "+r"(o.pa), "+r"(o.dsa), "+r"(o.qa), "+r"(o.doa));
        return o;
      };
      auto mma_s = [&](const Ops& o) {  // S^T = K Q^T
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma(tS, smem_desc_sw128(o.ka + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024),
                 smem_desc_sw128(o.qa + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024), kIdSq, kk > 0 ? 1u : 0u);
        tc_commit(s_full);
      };
      auto mma_dp = [&](const Ops& o) {  // dP^T = V dO^T
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma(tP, smem_desc_sw128(o.va + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024),
                 smem_desc_sw128(o.doa + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024), kIdSq, kk > 0 ? 1u : 0u);
        tc_commit(dp_full);
      };
      auto mma_dv = [&](const Ops& o, int it) {  // dV += P^T dO   (K = 128 queries)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma(tV, smem_desc_sw128(o.pa + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024),
                 smem_desc_sw128(o.doa + kk * 2048, 16384, 1024), kIdKV, (it > 0 || kk > 0) ? 1u : 0u);
        tc_commit(p_free);
      };
      auto mma_dk = [&](const Ops& o, int it) {  // dK += dS^T Q
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma(tK, smem_desc_sw128(o.dsa + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024),
                 smem_desc_sw128(o.qa + kk * 2048, 16384, 1024), kIdKV, (it > 0 || kk > 0) ? 1u : 0u);
      };
      auto mma_dq = [&](const Ops& o, int it) {  // dQ = dS K   (A = dS read MN-major, K = 128 keys)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma(tQ, smem_desc_sw128(o.dsa + kk * 2048, 16384, 1024),
                 smem_desc_sw128(o.ka + kk * 2048, 16384, 1024), kIdQ, kk > 0 ? 1u : 0u);
        tc_commit(dq_full);
        tc_commit(ds_free);
        tc_commit(q_empty0 + 8 * (it % STAGES));
      };
      auto q_ready = [&](int it) { return mbar_wait(q_full0 + 8 * (it % STAGES), (it / STAGES) & 1, status); };
      if constexpr (kAhead) {
        // S of the next query tile is issued before dK / dQ of this one, so the
        // compute warps find it ready when they finish dS; dP of the next tile
        // follows dQ.  Needs a second Q / dO stage and dQ in its own columns.
        if (ok && (ok = q_ready(0))) {
          tc_fence_after();
          const Ops o = ops(0);
          mma_s(o);
          mma_dp(o);
        }
#pragma unroll 1
        for (int it = 0; it < n_it && ok; ++it) {
          const uint32_t par = it & 1;
          const Ops o = ops(it);
          if (!(ok = mbar_wait(p_full, par, status))) break;
          tc_fence_after();
          mma_dv(o, it);
          const bool more = it + 1 < n_it;
          if (more) {
            if (!(ok = q_ready(it + 1) && mbar_wait(s_free, par, status))) break;
            tc_fence_after();
            mma_s(ops(it + 1));
          }
          if (!(ok = mbar_wait(ds_full, par, status))) break;
          tc_fence_after();
          mma_dk(o, it);
          if (!(ok = mbar_wait(dq_free, par ^ 1, status))) break;
          tc_fence_after();
          mma_dq(o, it);
          if (more) mma_dp(ops(it + 1));
        }
      } else {
#pragma unroll 1
        for (int it = 0; it < n_it && ok; ++it) {
          const uint32_t par = it & 1;
          const Ops o = ops(it);
          if (!(ok = q_ready(it) && mbar_wait(s_free, par ^ 1, status))) break;
          tc_fence_after();
          mma_s(o);
          if (!kOwnDq) {  // dQ of the previous tile lives in the dP^T columns
            if (!(ok = mbar_wait(dq_free, par ^ 1, status))) break;
            tc_fence_after();
          }
          mma_dp(o);
          if (!(ok = mbar_wait(p_full, par, status))) break;
          tc_fence_after();
          mma_dv(o, it);
          if (!(ok = mbar_wait(ds_full, par, status))) break;
          tc_fence_after();
          mma_dk(o, it);
          if (kOwnDq) {
            if (!(ok = mbar_wait(dq_free, par ^ 1, status))) break;
            tc_fence_after();
          }
          mma_dq(o, it);
        }
      }
      if (ok) tc_commit(acc_full);
    }
  } else {
    const int qd = warp & 3;
    const int part = (warp - 2) / 4;
    const int r = qd * 32 + lane;  // key row (S^T, dP^T, dK, dV) or query row (dQ)
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const float sl2 = scale * kLog2e;
    const int x = r % 8;  // swizzle phase of this row
    const int box = part / kPerBox;                       // dQ staging box of this part
    const int box_chunk = (part % kPerBox) * (kFill / 4);  // first 16-byte chunk of this part in a box row
    const uint32_t dq_box = sbase + S::dq_off + box * 16384, dq_row = row_base(dq_box, r);
    const uint32_t stg_free = stg_free0 + 8 * box, stg_full = stg_full0 + 8 * box;
    const bool leader = warp == 2 + 4 * part && part % kPerBox == 0 && lane == 0;  // issues this box's reduces
    uint32_t uses = 0;  // staging-box uses so far (mbarrier phase)
    uint32_t pk[kSCols / 2];  // this row of P^T as bf16 pairs: the values the dV MMA reads, reused for dS
    auto lse_of = [&](int it) { return sbase + S::st_off + (it % STAGES) * S::stage_bytes + 2 * S::tile; };
    // 32-column group c of this part: its bf16 row in a [128 x 64] swizzled atom
    auto col_of = [&](int c) { return part * kSCols + c * 32; };
    auto atom_row = [&](uint32_t off, int col0) { return row_base(sbase + off + (col0 / 64) * 16384, r); };
    // P^T = exp2(S^T * scale * log2e - lse * log2e), causal mask on the diagonal tile
    auto p_phase = [&](int it) -> bool {
      const uint32_t par = it & 1;
      bool ok = __all_sync(0xffffffffu, mbar_wait(s_full, par, status));
      if (ok && it > 0) ok = __all_sync(0xffffffffu, mbar_wait(p_free, par ^ 1, status));
      if (!ok) return false;
      tc_fence_after();
      const uint32_t st_lse = lse_of(it);  // float[128]
      const bool diag = it == 0;
#pragma unroll
      for (int c = 0; c < kSCols / 32; ++c) {
        const int col0 = col_of(c);
        float sv[32];
        tmem_ld_32(tS + lane_base + col0, sv);
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int qq = col0 + t;
          const float2 l2 = ld_shared_f2(st_lse + qq * 4);
          const float2 xs = fma2(make_float2(sv[t], sv[t + 1]), splat2(sl2), mul2(l2, splat2(-kLog2e)));
          float p0 = fast_exp2(xs.x);
          float p1 = fast_exp2(xs.y);
          if (diag && qq < r) p0 = 0.f;
          if (diag && qq + 1 < r) p1 = 0.f;
          pk[c * 16 + t / 2] = pack_bf16x2(p0, p1);
        }
        store_row_words(atom_row(S::p_off, col0), x, (col0 % 64) / 32, pk + c * 16);
      }
      tc_fence_before();
      mbar_arrive(s_free);
      fence_async_smem();
      mbar_arrive(p_full);
      return true;
    };
    // dS^T = scale * P^T (dP^T - delta)
    auto ds_phase = [&](int it) -> bool {
      const uint32_t par = it & 1;
      bool ok = __all_sync(0xffffffffu, mbar_wait(dp_full, par, status));
      if (ok && it > 0) ok = __all_sync(0xffffffffu, mbar_wait(ds_free, par ^ 1, status));
      if (!ok) return false;
      tc_fence_after();
      const uint32_t st_dl = lse_of(it) + 512;  // float[128]
#pragma unroll
      for (int c = 0; c < kSCols / 32; ++c) {
        const int col0 = col_of(c);
        float dv[32];
        tmem_ld_32(tP + lane_base + col0, dv);
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int qq = col0 + t;
          const float2 pp = unpack_bf16x2(pk[c * 16 + t / 2]);
          const float2 d2 = ld_shared_f2(st_dl + qq * 4);
          const float2 ds = mul2(mul2(splat2(scale), pp), sub2(make_float2(dv[t], dv[t + 1]), d2));
          dv[t] = ds.x;
          dv[t + 1] = ds.y;
        }
        store_row_bf16(atom_row(S::ds_off, col0), x, (col0 % 64) / 32, dv);
      }
      tc_fence_before();
      fence_async_smem();
      mbar_arrive(ds_full);
      return true;
    };
    // dQ_i rows (TMEM lane = query): TMEM -> registers (columns freed at
    // once) -> swizzled staging box -> one TMA reduce-add per 32 columns.
    auto flush = [&](int it) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(dq_full, it & 1, status))) return false;
      tc_fence_after();
      float qv[kDCols];
      if constexpr (kDCols == 16) {
        tmem_ld_16(tQ + lane_base + part * kDCols, qv);
      } else {
#pragma unroll
        for (int c = 0; c < kDCols / 32; ++c) tmem_ld_32(tQ + lane_base + part * kDCols + c * 32, qv + c * 32);
      }
      tc_fence_before();
      mbar_arrive(dq_free);
#pragma unroll
      for (int f = 0; f < kDCols / kFill; ++f, ++uses) {
        if (leader) {  // the box is free once the previous reduce has read it
          bulk_wait_read<0>();
          mbar_arrive(stg_free);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(stg_free, uses & 1, status))) return false;
#pragma unroll
        for (int k = 0; k < kFill / 4; ++k) {
          const float* v = qv + f * kFill + 4 * k;
          st_shared_v4(dq_row + (((box_chunk + k) ^ x) << 4), __float_as_uint(v[0]), __float_as_uint(v[1]),
                       __float_as_uint(v[2]), __float_as_uint(v[3]));
        }
        fence_async_smem();
        mbar_arrive(stg_full);
        bool staged = true;
        if (leader && (staged = mbar_wait(stg_full, uses & 1, status))) {
          tma_reduce_add_2d(&map_dq, dq_box, h * D + box * (kPerBox * kDCols) + f * 32, b * T + (j + it) * 128);
          bulk_commit();
        }
        if (!__all_sync(0xffffffffu, staged)) return false;
      }
      return true;
    };
    bool ok = true;
    if constexpr (kAhead) {
      // P of the next query tile is computed while dK / dQ of this one run
      ok = n_it > 0 && p_phase(0);
#pragma unroll 1
      for (int it = 0; it < n_it && ok; ++it) {
        ok = ds_phase(it) && (it + 1 >= n_it || p_phase(it + 1)) && flush(it);
      }
    } else {
#pragma unroll 1
      for (int it = 0; it < n_it && ok; ++it) ok = p_phase(it) && ds_phase(it) && flush(it);
    }
    if (leader) bulk_wait_all();  // dQ adds complete before the CTA exits
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, status));
    if (ok) {
      tc_fence_after();
      const long long row = static_cast<long long>(b) * T + j * 128 + r;
      __nv_bfloat16* dk = dqkv + row * 3 * C + C + h * D + part * kDCols;
      __nv_bfloat16* dv = dk + C;
      constexpr int kChunk = kDCols < 32 ? kDCols : 32;  // columns per TMEM load
      constexpr int kPer = kDCols / kChunk;
#pragma unroll 1
      for (int g = 0; g < 2 * kPer; ++g) {  // dK chunks, then dV chunks
        const int c = g % kPer;
        float kv[kChunk];
        const uint32_t src = (g < kPer ? tK : tV) + lane_base + part * kDCols + c * kChunk;
        if constexpr (kChunk == 16) tmem_ld_16(src, kv);
        else tmem_ld_32(src, kv);
        __nv_bfloat16* dst = (g < kPer ? dk : dv) + c * kChunk;
#pragma unroll
        for (int t = 0; t < kChunk; t += 8)
          *reinterpret_cast<uint4*>(dst + t) =
              make_uint4(pack_bf16x2(kv[t], kv[t + 1]), pack_bf16x2(kv[t + 2], kv[t + 3]),
                         pack_bf16x2(kv[t + 4], kv[t + 5]), pack_bf16x2(kv[t + 6], kv[t + 7]));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace fatc

// qkv: [B, T, 3*H*D] bf16 (row stride 3C, q|k|v thirds); o: [B, T, H*D]; lse: [B, H, T].
void flash_attn_fwd_tc(torch::Tensor qkv, torch::Tensor o, torch::Tensor lse, int64_t n_head, double scale,
                       torch::Tensor status) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3 && qkv.is_contiguous(),
              "qkv must be a contiguous CUDA bf16 [B, T, 3C] tensor");
  const int B = static_cast<int>(qkv.size(0)), T = static_cast<int>(qkv.size(1));
  const int C3 = static_cast<int>(qkv.size(2));
  const int H = static_cast<int>(n_head);
  const int D = C3 / 3 / H;
  TORCH_CHECK(D == 64 || D == 128, "tcgen05 attention supports head dim 64 or 128");
  c10::cuda::CUDAGuard g(qkv.device());
  CUtensorMap map = make_tma_2d_bf16(qkv.data_ptr(), C3, static_cast<uint64_t>(B) * T, C3, 64, 128);
  dim3 grid(B * H, (T + fatc::kQ - 1) / fatc::kQ);
  auto stream = at::cuda::getCurrentCUDAStream();
  auto run = [&](auto kern, uint32_t smem) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, fatc::kThreads, smem, stream>>>(map, reinterpret_cast<__nv_bfloat16*>(o.data_ptr()),
                                                 lse.data_ptr<float>(), H, T, static_cast<float>(scale),
                                                 status.data_ptr<int>());
  };
  static const bool single = std::getenv("MNB_ATTN_FWD_SINGLE") != nullptr;  // A/B switch for benchmarks
  // MNB_ATTN_POLY=1: half of the exponentials as exp2_poly (measured 12 %
  // slower at B16 H12 T1024 D64 than all on MUFU, so off by default)
  static const bool poly = std::getenv("MNB_ATTN_POLY") != nullptr;
  // MNB_ATTN_PACKED=1: f32x2 pairs in the softmax (measured 1-3 % slower than
  // scalar at B16 H12 T1024 D64, so off by default)
  static const bool packed = std::getenv("MNB_ATTN_PACKED") != nullptr;
  if (D == 64 && T % 256 == 0 && !single) {
    grid.y = T / 256;
    if (poly)
      run(fatc::fa_fwd_pp_kernel<true, false>, fatc::PPSmem::total);
    else if (packed)
      run(fatc::fa_fwd_pp_kernel<false, true>, fatc::PPSmem::total);
    else
      run(fatc::fa_fwd_pp_kernel<false, false>, fatc::PPSmem::total);
  } else if (D == 64) {
    run(fatc::fa_fwd_tc_kernel<64, 2>, fatc::Smem<64, 2>::total);
  } else {
    run(fatc::fa_fwd_tc_kernel<128, 2>, fatc::Smem<128, 2>::total);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward launch (delta and the zeroed fp32 dq accumulator are prepared by the
// caller, which also converts dq_acc afterwards): dqkv [B, T, 3C] receives dK
// and dV; qkv [B, T, 3C], dout [B, T, C] contiguous; T % 128 == 0.
void flash_attn_bwd_tc_launch(torch::Tensor qkv, torch::Tensor dout, torch::Tensor lse, torch::Tensor delta,
                              torch::Tensor dq_acc, torch::Tensor dqkv, int64_t n_head, double scale,
                              torch::Tensor status) {
  const int B = static_cast<int>(qkv.size(0)), T = static_cast<int>(qkv.size(1));
  const int C3 = static_cast<int>(qkv.size(2));
  const int H = static_cast<int>(n_head);
  const int C = C3 / 3;
  const int D = C / H;
  TORCH_CHECK(D == 64 || D == 128, "tcgen05 attention backward supports head dim 64 or 128");
  TORCH_CHECK(T % 128 == 0, "tcgen05 attention backward needs T % 128 == 0");
  TORCH_CHECK(qkv.is_contiguous() && dout.is_contiguous() && dqkv.is_contiguous(), "contiguous tensors");
  c10::cuda::CUDAGuard g(qkv.device());
  CUtensorMap mqkv = make_tma_2d_bf16(qkv.data_ptr(), C3, static_cast<uint64_t>(B) * T, C3, 64, 128);
  CUtensorMap mdo = make_tma_2d_bf16(dout.data_ptr(), C, static_cast<uint64_t>(B) * T, C, 64, 128);
  TORCH_CHECK(dq_acc.is_contiguous() && dq_acc.numel() == static_cast<int64_t>(B) * T * C, "dq_acc [B, T, C] fp32");
  CUtensorMap mdq = make_tma_2d_f32(dq_acc.data_ptr(), C, static_cast<uint64_t>(B) * T, C, 32, 128);
  dim3 grid(B * H, T / 128);
  auto stream = at::cuda::getCurrentCUDAStream();
  auto run = [&](auto kern, uint32_t smem, int parts) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, fatc::bwd_threads(parts), smem, stream>>>(
        mqkv, mdo, mdq, lse.data_ptr<float>(), delta.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), H, T, static_cast<float>(scale), status.data_ptr<int>());
  };
  // A/B switch for benchmarks: MNB_ATTN_BWD_PARTS=2 runs the 8-compute-warp kernel at D = 64
  static const char* parts_env = std::getenv("MNB_ATTN_BWD_PARTS");
  static const bool two_parts = parts_env != nullptr && parts_env[0] == '2';
  if (D == 64 && !two_parts) run(fatc::fa_bwd_tc_kernel<64, 2, 4>, fatc::BwdSmem<64, 2>::total, 4);
  else if (D == 64) run(fatc::fa_bwd_tc_kernel<64, 2, 2>, fatc::BwdSmem<64, 2>::total, 2);
  else run(fatc::fa_bwd_tc_kernel<128, 1, 2>, fatc::BwdSmem<128, 1>::total, 2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


// exp2_poly over a tensor (numerics test of the polynomial against exp2).
__global__ void exp2_poly_kernel(const float* x, float* y, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = fatc::exp2_poly(x[i]);
}

void exp2_poly_eval(torch::Tensor x, torch::Tensor y) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous() && y.sizes() == x.sizes() &&
                  y.scalar_type() == at::kFloat && y.is_contiguous(),
              "exp2_poly_eval: contiguous fp32 CUDA tensors of one shape");
  const long long n = x.numel();
  const int blocks = static_cast<int>(std::min<long long>((n + 255) / 256, 4096));
  exp2_poly_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(), y.data_ptr<float>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mnb
