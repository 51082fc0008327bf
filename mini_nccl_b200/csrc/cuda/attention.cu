// Causal flash attention, forward and backward, bf16 in / fp32 accumulate.
//
// Algorithm: FlashAttention-2 (Dao, 2023) -- tiles of 64 queries x 64 keys,
// online softmax in base 2 with the row max and sum kept in registers, the
// score tile reused in registers as the A operand of the P*V product, and a
// backward that walks key tiles with the queries as the inner loop,
// accumulating dK/dV in registers and dQ through fp32 vector atomics.  Fully
// masked tiles above the diagonal are never visited.
//
// Tensor-core path: warp-level mma.sync m16n8k16 (bf16 -> fp32) fed by
// ldmatrix from XOR-swizzled shared memory.
//
// Layout: q, k, v are [B, T, H*D] with an arbitrary row stride (so the three
// thirds of a fused QKV projection are used in place); o is [B, T, H*D]
// contiguous; lse is [B, H, T] fp32 (natural-log logsumexp of the scaled
// scores).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace mnb {

namespace fa {

constexpr int kTile = 64;     // queries per forward block / keys per backward block
constexpr int kThreads = 128;  // 4 warps
constexpr float kLog2e = 1.4426950408889634f;

MNB_DEVICE void mma_bf16(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
MNB_DEVICE void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
MNB_DEVICE void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
MNB_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill rows past the end of the sequence
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
MNB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
MNB_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Byte offset of 16-byte chunk `c` of row `r` in a [rows][D] bf16 tile whose
// chunks are XOR-swizzled by the row (conflict-free ldmatrix).
template <int D>
MNB_DEVICE uint32_t swz(int r, int c) {
  constexpr int chunks = D / 8;
  constexpr int mask = chunks >= 8 ? 7 : chunks - 1;
  return static_cast<uint32_t>((r * chunks + (c ^ (r & mask))) * 16);
}

// Copy a [64][D] tile (rows clipped to `valid_rows`) from global to shared.
template <int D>
MNB_DEVICE void load_tile(uint32_t sbase, const __nv_bfloat16* g, long long ld, int valid_rows) {
  constexpr int chunks = D / 8;
  for (int i = threadIdx.x; i < kTile * chunks; i += kThreads) {
    const int r = i / chunks, c = i % chunks;
    const bool ok = r < valid_rows;
    cp_async16(sbase + swz<D>(r, c), g + (ok ? r : 0) * ld + c * 8, ok);
  }
}

MNB_DEVICE uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads) fa_fwd_kernel(const __nv_bfloat16* __restrict__ q,
                                                          const __nv_bfloat16* __restrict__ k,
                                                          const __nv_bfloat16* __restrict__ v, long long ld_qkv,
                                                          __nv_bfloat16* __restrict__ o, float* __restrict__ lse,
                                                          int H, int T, float scale) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sQ = smem_u32(sm);
  const uint32_t sK = sQ + kTile * D * 2;
  const uint32_t sV = sK + kTile * D * 2;
  const int qt = gridDim.x - 1 - blockIdx.x;  // heaviest (longest causal) tiles first
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int q0 = qt * kTile;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, tg = lane % 4;
  const long long base = static_cast<long long>(b) * T * ld_qkv + static_cast<long long>(h) * D;

  load_tile<D>(sQ, q + base + q0 * ld_qkv, ld_qkv, T - q0);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();

  // Q fragments for this warp's 16 rows: D/16 k-chunks x 4 registers.
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kc = 0; kc < D / 16; ++kc) {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = kc * 2 + (lane >> 4);
    ldsm_x4(qf[kc], sQ + swz<D>(r, c));
  }

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const float sl2 = scale * kLog2e;
  const int row0 = q0 + warp * 16 + g;  // this thread's rows: row0 and row0 + 8

  const int n_kv = min(qt + 1, (T + kTile - 1) / kTile);
  for (int j = 0; j < n_kv; ++j) {
    const int k0 = j * kTile;
    __syncthreads();  // previous tile fully consumed
    load_tile<D>(sK, k + base + k0 * ld_qkv, ld_qkv, T - k0);
    load_tile<D>(sV, v + base + k0 * ld_qkv, ld_qkv, T - k0);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();

    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < D / 16; ++kc) {
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        // two key n-tiles (16 keys) x 16 d: matrices (keys n..n+7, d lo), (n, d hi), (n+8, lo), (n+8, hi)
        uint32_t kb[4];
        const int r = n * 8 + (lane & 7) + (lane >> 4) * 8;
        const int c = kc * 2 + ((lane >> 3) & 1);
        ldsm_x4(kb, sK + swz<D>(r, c));
        mma_bf16(s[n], qf[kc], kb);
        mma_bf16(s[n + 1], qf[kc], kb + 2);
      }
    }
    // scale, causal + length mask, online softmax (rows g and g+8 of this warp)
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = row0 + (e >> 1) * 8;
        const int col = k0 + n * 8 + tg * 2 + (e & 1);
        float x = s[n][e] * sl2;
        if (col > row || col >= T) x = -INFINITY;
        s[n][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      alpha[i] = (m_r[i] == -INFINITY) ? 0.f : exp2f(m_r[i] - mx[i]);
      m_r[i] = mx[i];
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        const float p = (s[n][e] == -INFINITY) ? 0.f : exp2f(s[n][e] - mm);
        s[n][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) l_r[i] = l_r[i] * alpha[i] + rs[i];
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      acc[dn][0] *= alpha[0];
      acc[dn][1] *= alpha[0];
      acc[dn][2] *= alpha[1];
      acc[dn][3] *= alpha[1];
    }
    // O += P V ; P (16 x 64) from registers, V (64 keys x D) via ldmatrix.trans
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t pa[4] = {pack2(s[2 * kc][0], s[2 * kc][1]), pack2(s[2 * kc][2], s[2 * kc][3]),
                        pack2(s[2 * kc + 1][0], s[2 * kc + 1][1]), pack2(s[2 * kc + 1][2], s[2 * kc + 1][3])};
#pragma unroll
      for (int dn = 0; dn < D / 8; dn += 2) {
        // matrices: (keys kc*16+0..7, d dn), (keys +8..15, d dn), (keys 0..7, d dn+1), (keys 8..15, d dn+1)
        uint32_t vb[4];
        const int r = kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dn + (lane >> 4);
        ldsm_x4_t(vb, sV + swz<D>(r, c));
        mma_bf16(acc[dn], pa, vb);
        mma_bf16(acc[dn + 1], pa, vb + 2);
      }
    }
  }
  // finalize: full row sums across the quad
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 1);
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 2);
  }
  const long long C = static_cast<long long>(H) * D;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int row = row0 + i * 8;
    if (row >= T) continue;
    const float inv = l_r[i] > 0.f ? 1.f / l_r[i] : 0.f;
    __nv_bfloat16* orow = o + (static_cast<long long>(b) * T + row) * C + h * D;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      *reinterpret_cast<uint32_t*>(orow + dn * 8 + tg * 2) = pack2(acc[dn][2 * i] * inv, acc[dn][2 * i + 1] * inv);
    }
    if (tg == 0) lse[(static_cast<long long>(b) * H + h) * T + row] = (m_r[i] + log2f(l_r[i])) / kLog2e;
  }
}

// ---------------------------------------------------------------------------
// backward preprocessing: Di = rowsum(dO * O)
// ---------------------------------------------------------------------------
template <int D>
__global__ void fa_bwd_dot_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                  float* __restrict__ delta, int H, int T, long long rows) {
  // delta[b, h, t] = sum_d O[b, t, h, d] * dO[b, t, h, d]; D / 8 lanes per row,
  // 16-byte loads, 32 * 8 / D rows per warp at a time.
  constexpr int LPR = D / 8;            // lanes per row
  constexpr int RPW = 32 / LPR;         // rows per warp pass
  const int lane = threadIdx.x % 32;
  const long long warp = blockIdx.x * (blockDim.x / 32LL) + threadIdx.x / 32;
  const long long r = warp * RPW + lane / LPR;  // r indexes (b, t, h)
  const int c = (lane % LPR) * 8;
  float s = 0.f;
  if (r < rows) {
    const uint4 a = *reinterpret_cast<const uint4*>(o + r * D + c);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + r * D + c);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = unpack_bf16x2(av[k]), y = unpack_bf16x2(gv[k]);
      s += x.x * y.x + x.y * y.y;
    }
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (r < rows && lane % LPR == 0) {
    const long long bt = r / H;
    const int h = static_cast<int>(r % H);
    const long long b = bt / T;
    const int t = static_cast<int>(bt % T);
    delta[(b * H + h) * T + t] = s;
  }
}

// ---------------------------------------------------------------------------
// backward: one block per (64-key tile, batch*head); 4 warps x 16 keys.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads) fa_bwd_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    long long ld_qkv, const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ delta, float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dk,
    __nv_bfloat16* __restrict__ dv, long long ld_dkv, int H, int T, float scale) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sK = smem_u32(sm);
  const uint32_t sV = sK + kTile * D * 2;
  const uint32_t sQ = sV + kTile * D * 2;
  const uint32_t sO = sQ + kTile * D * 2;                          // dO tile
  const uint32_t sS = sO + kTile * D * 2;                          // dS^T staging [64 keys][64 q] bf16
  float* sL = reinterpret_cast<float*>(sm + 4 * kTile * D * 2 + kTile * kTile * 2);  // lse*log2e [64]
  float* sDl = sL + kTile;                                                            // delta [64]

  const int kt = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int k0 = kt * kTile;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, tg = lane % 4;
  const long long base = static_cast<long long>(b) * T * ld_qkv + static_cast<long long>(h) * D;
  const long long C = static_cast<long long>(H) * D;
  const long long obase = static_cast<long long>(b) * T * C + static_cast<long long>(h) * D;
  const float sl2 = scale * kLog2e;

  load_tile<D>(sK, k + base + k0 * ld_qkv, ld_qkv, T - k0);
  load_tile<D>(sV, v + base + k0 * ld_qkv, ld_qkv, T - k0);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();

  // K and V fragments of this warp's 16 keys, as A operands.
  uint32_t kf[D / 16][4], vf[D / 16][4];
#pragma unroll
  for (int kc = 0; kc < D / 16; ++kc) {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = kc * 2 + (lane >> 4);
    ldsm_x4(kf[kc], sK + swz<D>(r, c));
    ldsm_x4(vf[kc], sV + swz<D>(r, c));
  }
  float dkacc[D / 8][4], dvacc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dkacc[i][e] = dvacc[i][e] = 0.f;

  const int key0 = k0 + warp * 16 + g;  // this thread's keys: key0, key0 + 8
  const int n_q = (T + kTile - 1) / kTile;
  for (int qt = kt; qt < n_q; ++qt) {
    const int q0 = qt * kTile;
    __syncthreads();
    load_tile<D>(sQ, q + base + q0 * ld_qkv, ld_qkv, T - q0);
    load_tile<D>(sO, dout + obase + q0 * C, C, T - q0);
    cp_async_commit();
    for (int i = threadIdx.x; i < kTile; i += kThreads) {
      const int qq = q0 + i;
      const long long li = (static_cast<long long>(b) * H + h) * T + qq;
      sL[i] = qq < T ? lse[li] * kLog2e : 0.f;
      sDl[i] = qq < T ? delta[li] : 0.f;
    }
    cp_async_wait_all();
    __syncthreads();

    // S^T (16 keys x 64 q) = K_w Q^T ; dP^T = V_w dO^T
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[n][e] = dpt[n][e] = 0.f;
#pragma unroll
    for (int kc = 0; kc < D / 16; ++kc) {
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t qb[4], ob[4];
        const int r = n * 8 + (lane & 7) + (lane >> 4) * 8;
        const int c = kc * 2 + ((lane >> 3) & 1);
        ldsm_x4(qb, sQ + swz<D>(r, c));
        ldsm_x4(ob, sO + swz<D>(r, c));
        mma_bf16(st[n], kf[kc], qb);
        mma_bf16(st[n + 1], kf[kc], qb + 2);
        mma_bf16(dpt[n], vf[kc], ob);
        mma_bf16(dpt[n + 1], vf[kc], ob + 2);
      }
    }
    // P^T and dS^T in place
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + (e >> 1) * 8;
        const int ql = n * 8 + tg * 2 + (e & 1);
        const int qq = q0 + ql;
        const bool live = qq >= key && qq < T && key < T;
        const float p = live ? exp2f(st[n][e] * sl2 - sL[ql]) : 0.f;
        st[n][e] = p;
        dpt[n][e] = p * (dpt[n][e] - sDl[ql]) * scale;
      }
    }
    // dV += P^T dO ; dK += dS^T Q   (A = [16 keys x 64 q] from registers, B = [64 q x D] via .trans)
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t pa[4] = {pack2(st[2 * kc][0], st[2 * kc][1]), pack2(st[2 * kc][2], st[2 * kc][3]),
                        pack2(st[2 * kc + 1][0], st[2 * kc + 1][1]), pack2(st[2 * kc + 1][2], st[2 * kc + 1][3])};
      uint32_t da[4] = {pack2(dpt[2 * kc][0], dpt[2 * kc][1]), pack2(dpt[2 * kc][2], dpt[2 * kc][3]),
                        pack2(dpt[2 * kc + 1][0], dpt[2 * kc + 1][1]),
                        pack2(dpt[2 * kc + 1][2], dpt[2 * kc + 1][3])};
#pragma unroll
      for (int dn = 0; dn < D / 8; dn += 2) {
        uint32_t ob[4], qb[4];
        const int r = kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dn + (lane >> 4);
        ldsm_x4_t(ob, sO + swz<D>(r, c));
        ldsm_x4_t(qb, sQ + swz<D>(r, c));
        mma_bf16(dvacc[dn], pa, ob);
        mma_bf16(dvacc[dn + 1], pa, ob + 2);
        mma_bf16(dkacc[dn], da, qb);
        mma_bf16(dkacc[dn + 1], da, qb + 2);
      }
    }
    // stage dS^T (bf16) so dQ = dS K can read it transposed
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int kr = warp * 16 + g + hh * 8;  // key row within the tile
        const int qc = n * 8 + tg * 2;          // query column
        const uint32_t off = static_cast<uint32_t>((kr * 8 + ((qc / 8) ^ (kr & 7))) * 16 + (qc % 8) * 2);
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(sS + off), "r"(pack2(dpt[n][2 * hh], dpt[n][2 * hh + 1])));
      }
    }
    __syncthreads();
    // dQ (64 q x D) = dS (64 q x 64 keys) K (64 keys x D); warp w computes q rows 16w..16w+15
    {
      float dq[D / 8][4];
#pragma unroll
      for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kc = 0; kc < 4; ++kc) {
        // A fragment of dS rows (q) 16w.., cols (keys) 16kc..: transpose of staged [key][q]
        uint32_t aa[4];
        {
          const int kr = kc * 16 + (lane & 7) + (lane >> 4) * 8;  // key row in staging
          const int qc = warp * 2 + ((lane >> 3) & 1);            // 16-byte chunk of q columns
          ldsm_x4_t(aa, sS + static_cast<uint32_t>((kr * 8 + (qc ^ (kr & 7))) * 16));
        }
#pragma unroll
        for (int dn = 0; dn < D / 8; dn += 2) {
          uint32_t kb[4];
          const int r = kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = dn + (lane >> 4);
          ldsm_x4_t(kb, sK + swz<D>(r, c));
          mma_bf16(dq[dn], aa, kb);
          mma_bf16(dq[dn + 1], aa, kb + 2);
        }
      }
#pragma unroll
      for (int dn = 0; dn < D / 8; ++dn) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int qq = q0 + warp * 16 + g + hh * 8;
          if (qq < T) {
            float* dst = dq_acc + ((static_cast<long long>(b) * T + qq) * H + h) * D + dn * 8 + tg * 2;
            atomicAdd(reinterpret_cast<float2*>(dst), make_float2(dq[dn][2 * hh], dq[dn][2 * hh + 1]));
          }
        }
      }
    }
  }
  // write dK, dV for this warp's 16 keys
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int key = key0 + i * 8;
    if (key >= T) continue;
    __nv_bfloat16* dkr = dk + (static_cast<long long>(b) * T + key) * ld_dkv + static_cast<long long>(h) * D;
    __nv_bfloat16* dvr = dv + (static_cast<long long>(b) * T + key) * ld_dkv + static_cast<long long>(h) * D;
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      *reinterpret_cast<uint32_t*>(dkr + dn * 8 + tg * 2) = pack2(dkacc[dn][2 * i], dkacc[dn][2 * i + 1]);
      *reinterpret_cast<uint32_t*>(dvr + dn * 8 + tg * 2) = pack2(dvacc[dn][2 * i], dvacc[dn][2 * i + 1]);
    }
  }
}

__global__ void fa_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, long long ld_dq,
                                     int HD, long long rows) {
  // 8 values per thread: two 16-byte loads, one 16-byte store (HD % 8 == 0)
  const long long n8 = rows * HD / 8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = 8 * i;
    const long long r = e / HD;
    const int c = static_cast<int>(e % HD);
    const float4 a = reinterpret_cast<const float4*>(acc)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(acc)[2 * i + 1];
    *reinterpret_cast<uint4*>(dq + r * ld_dq + c) =
        make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
  }
}

}  // namespace fa

static void check_qkv(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3 && t.stride(2) == 1, n,
              " must be a CUDA bf16 [B, T, H*D] tensor with unit inner stride");
}

// o: [B, T, H*D] contiguous; lse: [B, H, T] fp32
void flash_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse,
                    int64_t n_head, double scale) {
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  TORCH_CHECK(q.stride(1) == k.stride(1) && q.stride(1) == v.stride(1) && q.stride(0) == q.size(1) * q.stride(1),
              "q, k, v must share one row stride");
  const int B = static_cast<int>(q.size(0)), T = static_cast<int>(q.size(1));
  const int H = static_cast<int>(n_head);
  const int D = static_cast<int>(q.size(2) / H);
  c10::cuda::CUDAGuard g(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid((T + fa::kTile - 1) / fa::kTile, B * H);
  const long long ld = q.stride(1);
  auto run = [&](auto kern, int d) {
    const size_t smem = 3 * fa::kTile * d * 2;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, fa::kThreads, smem, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), ld, reinterpret_cast<__nv_bfloat16*>(o.data_ptr()),
        lse.data_ptr<float>(), H, T, static_cast<float>(scale));
  };
  if (D == 64) run(fa::fa_fwd_kernel<64>, 64);
  else if (D == 128) run(fa::fa_fwd_kernel<128>, 128);
  else if (D == 32) run(fa::fa_fwd_kernel<32>, 32);
  else TORCH_CHECK(false, "head dim must be 32, 64 or 128, got ", D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dq/dk/dv: [B, T, H*D] views (row stride ld_dqkv, e.g. thirds of a fused QKV
// gradient).  dq_acc: fp32 [B, T, H*D] scratch, delta: fp32 [B, H, T] scratch.
void flash_attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc,
                    torch::Tensor delta, int64_t n_head, double scale) {
  check_qkv(q, "q");
  check_qkv(dq, "dq");
  TORCH_CHECK(dout.is_contiguous() && o.is_contiguous(), "o and dout must be contiguous");
  TORCH_CHECK(dk.stride(1) == dv.stride(1), "dk and dv must share one row stride");
  const int B = static_cast<int>(q.size(0)), T = static_cast<int>(q.size(1));
  const int H = static_cast<int>(n_head);
  const int HD = static_cast<int>(q.size(2));
  const int D = HD / H;
  c10::cuda::CUDAGuard g(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const long long rows = static_cast<long long>(B) * T * H;
  dq_acc.zero_();
  auto dot = [&](auto kern) {
    const long long warps = (rows * D / 8 + 31) / 32;  // D/8 lanes per row
    kern<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        delta.data_ptr<float>(), H, T, rows);
  };
  auto run = [&](auto kern, int d) {
    const size_t smem = 4 * fa::kTile * d * 2 + fa::kTile * fa::kTile * 2 + 2 * fa::kTile * 4;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    dim3 grid((T + fa::kTile - 1) / fa::kTile, B * H);
    kern<<<grid, fa::kThreads, smem, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), q.stride(1),
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), lse.data_ptr<float>(), delta.data_ptr<float>(),
        dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), dk.stride(1), H, T, static_cast<float>(scale));
  };
  if (D == 64) {
    dot(fa::fa_bwd_dot_kernel<64>);
    run(fa::fa_bwd_kernel<64>, 64);
  } else if (D == 128) {
    dot(fa::fa_bwd_dot_kernel<128>);
    run(fa::fa_bwd_kernel<128>, 128);
  } else if (D == 32) {
    dot(fa::fa_bwd_dot_kernel<32>);
    run(fa::fa_bwd_kernel<32>, 32);
  } else {
    TORCH_CHECK(false, "head dim must be 32, 64 or 128");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const long long n2 = rows * D / 8;
  fa::fa_dq_convert_kernel<<<static_cast<unsigned>(std::min<long long>((n2 + 255) / 256, 148 * 16)), 256, 0,
                             stream>>>(dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()),
                                       dq.stride(1), HD, static_cast<long long>(B) * T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void flash_attn_bwd_tc_launch(torch::Tensor qkv, torch::Tensor dout, torch::Tensor lse, torch::Tensor delta,
                              torch::Tensor dq_acc, torch::Tensor dqkv, int64_t n_head, double scale,
                              torch::Tensor status);

// tcgen05 backward: qkv / dqkv [B, T, 3C] contiguous, o / dout [B, T, C]
// contiguous, lse [B, H, T]; dq_acc [B, T, C] fp32 and delta [B, H, T] fp32
// are scratch.  T % 128 == 0, head dim 64 or 128.
void flash_attn_bwd_tc(torch::Tensor qkv, torch::Tensor o, torch::Tensor dout, torch::Tensor lse, torch::Tensor dqkv,
                       torch::Tensor dq_acc, torch::Tensor delta, int64_t n_head, double scale, torch::Tensor status) {
  TORCH_CHECK(o.is_contiguous() && dout.is_contiguous(), "o and dout must be contiguous");
  const int B = static_cast<int>(qkv.size(0)), T = static_cast<int>(qkv.size(1));
  const int H = static_cast<int>(n_head);
  const int C = static_cast<int>(qkv.size(2)) / 3;
  const int D = C / H;
  c10::cuda::CUDAGuard g(qkv.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const long long rows = static_cast<long long>(B) * T * H;
  C10_CUDA_CHECK(cudaMemsetAsync(dq_acc.data_ptr(), 0, dq_acc.numel() * sizeof(float), stream));
  auto dot = [&](auto kern) {
    const long long warps = (rows * D / 8 + 31) / 32;  // D/8 lanes per row
    kern<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        delta.data_ptr<float>(), H, T, rows);
  };
  if (D == 64) dot(fa::fa_bwd_dot_kernel<64>);
  else if (D == 128) dot(fa::fa_bwd_dot_kernel<128>);
  else TORCH_CHECK(false, "tcgen05 attention backward supports head dim 64 or 128");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  flash_attn_bwd_tc_launch(qkv, dout, lse, delta, dq_acc, dqkv, n_head, scale, status);
  const long long n2 = rows * D / 8;
  fa::fa_dq_convert_kernel<<<static_cast<unsigned>(std::min<long long>((n2 + 255) / 256, 148 * 16)), 256, 0,
                             stream>>>(dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
                                       3LL * C, C, static_cast<long long>(B) * T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mnb
