// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The backward on the tensor cores: dQ, dK, dV of O = softmax(Q K^T * scale) V from dO, the
// forward's L and the prep kernel's D, written into ONE [b, s, 3, h, 64] buffer -- the same
// contract as bwd_ffma.cu (the reference's fattn_bwd_f32_d64, kernels/fused_attn.cu:213-426), with
// the five products on tcgen05.mma and fp32 from split bf16 parts as in fwd_tc.cu: every fp32
// operand x = x0 + x1 + x2 (three bf16), A B = A0B0 + (A0B1 + A1B0 + A0B2 + A1B1 + A2B0), every
// product in one TMEM accumulator that starts fresh every window of 64 reduction elements and
// takes the small products of the window's K-steps first and its A0B0 steps last; each window's
// sum is added in fp32 registers, round-to-nearest.
//
// Block: 512 threads own a key block of KB = 128 keys of one (batch, head) and walk its query
// tiles of QT = 64. Thread (warp w, lane l) owns key row 32 (w % 4) + l -- its TMEM lane -- and
// the 16 columns of group w / 4. Per query tile, with thread 0 issuing every MMA:
//   S^T  = K Q^T      A: K parts (K-major)      B: Q parts (K-major)        -> TMEM 0
//   dP^T = V dO^T     A: V parts                B: dO parts                 -> TMEM 64
//   the threads form P^T = exp(S^T * scale - L) (masked) and dS^T = P^T o (dP^T - D), put P^T's
//   parts into TMEM (the A operand of dV, over columns 0-95) and dS^T's into shared memory;
//   dV  += P^T dO     A: P^T parts in TMEM      B: dO parts read MN-major   -> TMEM 128
//   dK  += dS^T Q     A: dS^T parts (K-major)   B: Q parts read MN-major    -> TMEM 192
//   dQ_t = dS K       A: dS^T parts read MN-major (M = 64 queries)  B: K parts read MN-major
//                     keys 0-63 -> TMEM 256, keys 64-127 -> TMEM 320 (two windows)
//   dV and dK fold into fp32 registers per tile; the tile's dQ partial goes to the workspace and
//   the block that finishes last for its (batch, head) sums the partials in key-block order
//   (the no-wait path of bwd_ffma.cu: bit-identical for every schedule).
// S^T takes its six products in the forward kernel's order (A and B swapped), so the scores match
// fwd_tc.cu's and the recomputed P matches the forward's L.
//
// Every mbarrier wait is bounded; an expired wait sets the workspace error flag
// (cfa_bwd_status reads it) and the block writes nothing.
#include <cuda_bf16.h>

#include "cfa_common.cuh"
#include "cfa_internal.h"
#include "cfa_tc.cuh"

namespace cfa {
namespace {

constexpr int KB = 128;   // keys per block: MMA M of S^T, dP^T, dV, dK
constexpr int QT = 64;    // queries per tile: MMA N of S^T, dP^T; M of dQ
constexpr int NT = 512;   // threads
constexpr int PART_K = KB * 64 * 2;  // one bf16 part of a [128][64] operand
constexpr int PART_Q = QT * 64 * 2;  // one bf16 part of a [64][64] operand
constexpr int OFF_K = 0;                      // K parts [128 keys][64 d]
constexpr int OFF_V = OFF_K + 3 * PART_K;     // V parts [128 keys][64 d]
constexpr int OFF_Q = OFF_V + 3 * PART_K;     // Q parts [64 q][64 d]
constexpr int OFF_DO = OFF_Q + 3 * PART_Q;    // dO parts [64 q][64 d]
constexpr int OFF_DS = OFF_DO + 3 * PART_Q;   // dS^T parts [128 keys][64 q] (first: K staged)
constexpr int OFF_ST = OFF_DS + 3 * PART_K;   // staging: next Q, dO (fp32; first: V staged)
constexpr int OFF_LD = OFF_ST + 2 * QT * 64 * 4;  // L, D of two tiles: float [2][2][64]
constexpr int OFF_BAR = OFF_LD + 2 * 2 * QT * 4;  // mbarriers A (S, dP), B (dV, dK, dQ); TMEM base
constexpr int SMEM = OFF_BAR + 32;
constexpr int SMEM_ALLOC = SMEM + 1024;
constexpr uint32_t TMEM_COLS = 512;
static_assert(SMEM_ALLOC <= 232448, "shared memory per block");

__device__ __forceinline__ uint32_t kmaj_off(int row, int kc) {
  return static_cast<uint32_t>((((row >> 3) * 8 + kc) << 7) + ((row & 7) << 4));
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}

// x[0..7] -> three rows of 8 bf16 parts (x = p0 + p1 + p2 + below 2^-24 relative).
__device__ __forceinline__ void split8(const float (&x)[8], uint4& p0, uint4& p1, uint4& p2) {
  uint32_t a[4], b[4], c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float x0 = x[2 * i], x1 = x[2 * i + 1];
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    const float r0 = x0 - hf.x, r1 = x1 - hf.y;
    const __nv_bfloat162 m = __floats2bfloat162_rn(r0, r1);
    const float2 mf = __bfloat1622float2(m);
    const __nv_bfloat162 l = __floats2bfloat162_rn(r0 - mf.x, r1 - mf.y);
    a[i] = bf2_bits(h);
    b[i] = bf2_bits(m);
    c[i] = bf2_bits(l);
  }
  p0 = make_uint4(a[0], a[1], a[2], a[3]);
  p1 = make_uint4(b[0], b[1], b[2], b[3]);
  p2 = make_uint4(c[0], c[1], c[2], c[3]);
}

__device__ __forceinline__ void store_parts(unsigned char* base, int part_bytes, uint32_t off,
                                            const float (&x)[8]) {
  uint4 p0, p1, p2;
  split8(x, p0, p1, p2);
  *reinterpret_cast<uint4*>(base + off) = p0;
  *reinterpret_cast<uint4*>(base + part_bytes + off) = p1;
  *reinterpret_cast<uint4*>(base + 2 * part_bytes + off) = p2;
}

// Row items (row r, elements 8 kc .. 8 kc + 7): item c takes row 8 (c / 64) + c % 8 and chunk
// (c / 8) % 8 (a quarter-warp writes 8 rows of one chunk: 8 bank groups). Every thread copies
// (cp.async) the fp32 chunks it splits into slots of its own: slot j of thread t at
// (j * NT + t) * 16 bytes.
__device__ __forceinline__ void row_item(int c, int& r, int& kc) {
  r = 8 * (c >> 6) + (c & 7);
  kc = (c >> 3) & 7;
}

__device__ __forceinline__ void stage_row_item(unsigned char* st, int slot, int c, const float* src,
                                               int64_t stride, int r0, int seq) {
  int r, kc;
  row_item(c, r, kc);
  const bool ok = r0 + r < seq;
  const float* g = src + static_cast<int64_t>(ok ? r0 + r : 0) * stride + 8 * kc;
  cp_async16(st + 16 * ((2 * slot) * NT + threadIdx.x), g, ok ? 16 : 0);
  cp_async16(st + 16 * ((2 * slot + 1) * NT + threadIdx.x), g + 4, ok ? 16 : 0);
}

__device__ __forceinline__ void split_row_item(unsigned char* parts, int part_bytes,
                                               const unsigned char* st, int slot, int c) {
  int r, kc;
  row_item(c, r, kc);
  const float4 u = *reinterpret_cast<const float4*>(st + 16 * ((2 * slot) * NT + threadIdx.x));
  const float4 v = *reinterpret_cast<const float4*>(st + 16 * ((2 * slot + 1) * NT + threadIdx.x));
  const float x[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
  store_parts(parts, part_bytes, kmaj_off(r, kc), x);
}

// MMA with the A operand in TMEM (lane r = row r; a K step of 16 bf16 in 8 columns of packed
// pairs, the even element in the low half).
__device__ __forceinline__ void mma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// One window: six split products over STEPS K-steps into the fresh accumulator `d`; descriptors
// advance by A_STEP / B_STEP bytes per step and by A_PART / B_PART bytes per part. Part pairs
// (P0(p), P1(p)) -- the small (0, 1), (1, 0), (0, 2), (1, 1), (2, 0) of every step, then the
// (0, 0) of every step -- or, SWAP, (P1(p), P0(p)): the order in which the forward forms its
// products when A and B trade places.
__host__ __device__ constexpr int P0(int p) { return p == 2 || p == 4 ? 1 : (p == 5 ? 2 : 0); }
__host__ __device__ constexpr int P1(int p) { return p == 1 || p == 4 ? 1 : (p == 3 ? 2 : 0); }
template <int STEPS, int A_PART, int B_PART, int A_STEP, int B_STEP, bool SWAP>
__device__ __forceinline__ void issue6(uint32_t d, uint64_t ad0, uint64_t bd0, uint32_t idesc) {
#pragma unroll
  for (int ks = 0; ks < STEPS; ++ks)
#pragma unroll
    for (int p = 1; p < 6; ++p) {
      const int pa = SWAP ? P1(p) : P0(p), pb = SWAP ? P0(p) : P1(p);
      tc::mma_bf16(d, ad0 + static_cast<uint64_t>((pa * A_PART + A_STEP * ks) >> 4),
                   bd0 + static_cast<uint64_t>((pb * B_PART + B_STEP * ks) >> 4), idesc,
                   ks > 0 || p > 1);
    }
#pragma unroll
  for (int ks = 0; ks < STEPS; ++ks)
    tc::mma_bf16(d, ad0 + static_cast<uint64_t>((A_STEP * ks) >> 4),
                 bd0 + static_cast<uint64_t>((B_STEP * ks) >> 4), idesc, 1);
}

template <bool CAUSAL>
__global__ void __launch_bounds__(NT, 1) bwd_tc_kernel(const BwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* Kp = sm + OFF_K;
  unsigned char* Vp = sm + OFF_V;
  unsigned char* Qp = sm + OFF_Q;
  unsigned char* dOp = sm + OFF_DO;
  unsigned char* dSp = sm + OFF_DS;
  unsigned char* st = sm + OFF_ST;
  float* ld = reinterpret_cast<float*>(sm + OFF_LD);  // [buf][0: L, 1: D][64]
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* bar_b = bar_a + 1;
  uint32_t* tbase_p = reinterpret_cast<uint32_t*>(bar_a + 2);
  int* s_int = reinterpret_cast<int*>(bar_a + 3);

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int row = 32 * (w & 3) + lane;  // key row: TMEM lane
  const int cg = w >> 2;                // column group: 16 queries (S, dP) or dims (dV, dK, dQ)
  const int S = a.S;
  const int nkb = a.n_kblocks;
  // (b, h)-major: a (b, h)'s key blocks run side by side and its last one finishes early.
  const int kb = static_cast<int>(blockIdx.x) % nkb;
  const int bh = static_cast<int>(blockIdx.x) / nkb;
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kb * KB;
  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* kp = a.k + b * a.k_sb + h * a.k_sh;
  const float* vp = a.v + b * a.v_sb + h * a.v_sh;
  const float* gp = a.d_o + b * a.do_sb + h * a.do_sh;
  const float* lp = a.lse + static_cast<int64_t>(bh) * S;
  const float* dp = a.dsum + static_cast<int64_t>(bh) * S;
  const int n_tiles = (S + QT - 1) / QT;
  const int t_begin = CAUSAL ? k0 / QT : 0;  // queries before the block's first key see none

  if (tid == 0) {
    tc::mbar_init(bar_a, 1);
    tc::mbar_init(bar_b, 1);
    tc::fence_mbar_init();
  }
  if (w == 0) {
    tc::tmem_alloc(tbase_p, TMEM_COLS);
    tc::tmem_relinquish();
  }
  griddep_launch_dependents();

  // Q, dO, L, D of tile t into this thread's staging slots (Q: slots 0-1, dO: 2-3 of the staging
  // area) and L / D buffer `buf` (threads 0-127).
  auto stage_tile = [&](int t, int buf) {
    const int q0 = t * QT;
    stage_row_item(st, 0, tid, qp, a.q_ss, q0, S);
    stage_row_item(st, 1, tid, gp, a.do_ss, q0, S);
    if (tid < 2 * QT) {
      const int r = tid & 63, i = q0 + r;
      const bool ok = i < S;
      cp_async4(ld + buf * 128 + (tid < QT ? 0 : QT) + r, (tid < QT ? lp : dp) + (ok ? i : 0),
                ok ? 4 : 0);
    }
  };
  auto split_tile = [&]() {
    split_row_item(Qp, PART_Q, st, 0, tid);
    split_row_item(dOp, PART_Q, st, 1, tid);
  };

  // Prologue: K (staged in the dS^T buffer), V (in the staging area) and the first query tile.
  // K and V are caller inputs; L, D and the cleared counters come after the prep kernel's wait.
  stage_row_item(dSp, 0, tid, kp, a.k_ss, k0, S);
  stage_row_item(dSp, 1, tid + NT, kp, a.k_ss, k0, S);
  stage_row_item(st, 0, tid, vp, a.v_ss, k0, S);
  stage_row_item(st, 1, tid + NT, vp, a.v_ss, k0, S);
  cp_async_commit();
  cp_async_wait_all();
  split_row_item(Kp, PART_K, dSp, 0, tid);
  split_row_item(Kp, PART_K, dSp, 1, tid + NT);
  split_row_item(Vp, PART_K, st, 0, tid);
  split_row_item(Vp, PART_K, st, 1, tid + NT);
  __syncthreads();  // staging free
  griddep_wait();   // L, D, the cleared counters: the prep kernel's writes
  if (t_begin < n_tiles) stage_tile(t_begin, 0);
  cp_async_commit();
  cp_async_wait_all();
  split_tile();
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  const uint32_t tbase = *tbase_p;
  const uint32_t lane_sel = static_cast<uint32_t>(32 * (w & 3)) << 16;
  const uint32_t id128 = tc::idesc_f32acc(1, KB, QT);           // M 128, N 64, both K-major
  const uint32_t id_dv = id128 | (1u << 16);                     // B MN-major
  const uint32_t id_dq = tc::idesc_f32acc(1, QT, 64) | (1u << 15) | (1u << 16);  // M 64, A, B MN
  const uint32_t sK = tc::smem_u32(Kp), sV = tc::smem_u32(Vp), sQ = tc::smem_u32(Qp),
                 sO = tc::smem_u32(dOp), sS = tc::smem_u32(dSp);

  float dv[16], dk[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) dv[c] = dk[c] = 0.0f;
  bool err = false;
  const int key = k0 + row;

  int n = 0;  // tiles done: the mbarrier phase
  for (int t = t_begin; t < n_tiles; ++t, ++n) {
    const int q0 = t * QT, buf = n & 1;
    // (1) S^T and dP^T.
    if (tid == 0) {
      // S^T in the forward's product order (its pairs (Q i, K j) as (K j, Q i)).
      issue6<4, PART_K, PART_Q, 256, 256, true>(tbase, tc::desc_kmajor(sK, 128, 1024),
                                                tc::desc_kmajor(sQ, 128, 1024), id128);
      issue6<4, PART_K, PART_Q, 256, 256, false>(tbase + 64, tc::desc_kmajor(sV, 128, 1024),
                                                 tc::desc_kmajor(sO, 128, 1024), id128);
      tc::commit(bar_a);
    }
    // (2) the next tile travels.
    if (t + 1 < n_tiles) stage_tile(t + 1, buf ^ 1);
    cp_async_commit();
    // (3) P^T and dS^T for this thread's 16 queries.
    err |= !tc::mbar_wait(bar_a, n & 1, WAIT_TIMEOUT_NS);
    tc::fence_after_sync();
    const float* Lt = ld + buf * 128;
    const float* Dt = Lt + QT;
    const bool edge = (q0 + QT > S) || (k0 + KB > S) || (CAUSAL && k0 + KB - 1 > q0);
    float pr[16];
#pragma unroll
    for (int h8 = 0; h8 < 2; ++h8) {
      const uint32_t col = 16 * cg + 8 * h8;
      float sb[8], gb[8];
      tmem_ld8(tbase + lane_sel + col, sb);
      tmem_ld8(tbase + lane_sel + 64 + col, gb);
      tc::tmem_wait_ld();
      float ds[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int ql = col + u, qi = q0 + ql;
        // P = e^(s * scale - L), one rounding of the argument (as bwd_ffma.cu).
        float p = expf(fmaf(sb[u], a.scale, -Lt[ql]));
        if (edge && !(qi < S && key < S && !(CAUSAL && key > qi))) p = 0.0f;
        pr[8 * h8 + u] = p;
        ds[u] = p * (gb[u] - Dt[ql]);
      }
      store_parts(dSp, PART_K, kmaj_off(row, 2 * cg + h8), ds);
    }
    // (4) P^T's parts over columns 0-95, once every thread has read S^T and dP^T.
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    {
      uint4 lo[3], hi[3];
      float x0[8], x1[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        x0[u] = pr[u];
        x1[u] = pr[8 + u];
      }
      split8(x0, lo[0], lo[1], lo[2]);
      split8(x1, hi[0], hi[1], hi[2]);
#pragma unroll
      for (int pt = 0; pt < 3; ++pt) {
        const uint32_t v[8] = {lo[pt].x, lo[pt].y, lo[pt].z, lo[pt].w,
                               hi[pt].x, hi[pt].y, hi[pt].z, hi[pt].w};
        tmem_st8(tbase + lane_sel + 32 * pt + 8 * cg, v);
      }
      tc::tmem_wait_st();
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // (5) dV, dK, dQ.
    if (tid == 0) {
      const uint64_t bo_mn = tc::desc_kmajor(sO, 1024, 128);  // dO as B, MN-major (N = d)
      const uint64_t bq_mn = tc::desc_kmajor(sQ, 1024, 128);  // Q as B, MN-major
      const uint64_t bk_mn = tc::desc_kmajor(sK, 1024, 128);  // K as B, MN-major (K = keys)
      const uint64_t as_k = tc::desc_kmajor(sS, 128, 1024);   // dS^T as A, K-major
      const uint64_t as_mn = tc::desc_kmajor(sS, 1024, 128);  // dS^T as A, MN-major (M = q)
      // dV: P^T part i of K-step ks at TMEM column 32 i + 8 ks; the same pair order as issue6.
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int p = 1; p < 6; ++p)
          mma_bf16_tmem_a(tbase + 128, tbase + 32 * P0(p) + 8 * ks,
                          bo_mn + static_cast<uint64_t>((P1(p) * PART_Q + 2048 * ks) >> 4), id_dv,
                          ks > 0 || p > 1);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_bf16_tmem_a(tbase + 128, tbase + 8 * ks,
                        bo_mn + static_cast<uint64_t>((2048 * ks) >> 4), id_dv, 1);
      issue6<4, PART_K, PART_Q, 256, 2048, false>(tbase + 192, as_k, bq_mn, id_dv);
      // dQ: keys 0-63 and 64-127 (four K-steps each, 8192 bytes apart in both operands).
      issue6<4, PART_K, PART_K, 2048, 2048, false>(tbase + 256, as_mn, bk_mn, id_dq);
      issue6<4, PART_K, PART_K, 2048, 2048, false>(tbase + 320, as_mn + (8192 >> 4),
                                                   bk_mn + (8192 >> 4), id_dq);
      tc::commit(bar_b);
    }
    // (6) Fold dV, dK; write the dQ partial; the next tile's Q, dO into their parts.
    cp_async_wait_all();
    err |= !tc::mbar_wait(bar_b, n & 1, WAIT_TIMEOUT_NS);
    tc::fence_after_sync();
    {
      float xb[16], xs[16];
      tc::tmem_ld16(tbase + lane_sel + 128 + 16 * cg, xb);
      tc::tmem_ld16(tbase + lane_sel + 192 + 16 * cg, xs);
      tc::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        dv[c] += xb[c];
        dk[c] += xs[c];
      }
      // dQ (M = 64): query row 16 (w % 4) + lane in lanes 0-15 of each quarter; the two windows.
      tc::tmem_ld16(tbase + lane_sel + 256 + 16 * cg, xb);
      tc::tmem_ld16(tbase + lane_sel + 320 + 16 * cg, xs);
      tc::tmem_wait_ld();
      const int qi = q0 + 16 * (w & 3) + lane;
      if (lane < 16 && qi < S && !err) {
        float* dst = a.dq_part + ((static_cast<int64_t>(bh) * nkb + kb) * S + qi) * 64 + 16 * cg;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
          __stcg(reinterpret_cast<float4*>(dst) + c4,
                 make_float4(xb[4 * c4] + xs[4 * c4], xb[4 * c4 + 1] + xs[4 * c4 + 1],
                             xb[4 * c4 + 2] + xs[4 * c4 + 2], xb[4 * c4 + 3] + xs[4 * c4 + 3]));
      }
    }
    if (t + 1 < n_tiles) split_tile();
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  cp_async_wait_all();

  if (__syncthreads_or(err)) {
    if (tid == 0) atomicExch(a.err, CFA_ERR_TIMEOUT);
  } else {
    // dV into slot 2, dK * scale into slot 1 of dqkv [b, s, 3, h, 64].
    if (key < S) {
      const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * 64;
      float* base = a.dqkv + (static_cast<int64_t>(b) * S + key) * row_stride + h * 64 + 16 * cg;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        reinterpret_cast<float4*>(base + 2 * a.H * 64)[c4] =
            make_float4(dv[4 * c4], dv[4 * c4 + 1], dv[4 * c4 + 2], dv[4 * c4 + 3]);
        reinterpret_cast<float4*>(base + a.H * 64)[c4] =
            make_float4(dk[4 * c4] * a.scale, dk[4 * c4 + 1] * a.scale, dk[4 * c4 + 2] * a.scale,
                        dk[4 * c4 + 3] * a.scale);
      }
    }
    // The last of the (b, h)'s key blocks to finish sums its dQ partials in key-block order.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_int[0] = atomicAdd(a.turn + bh, 1);
    __syncthreads();
    if (s_int[0] == nkb - 1) {
      __threadfence();
      const float* part = a.dq_part + static_cast<int64_t>(bh) * nkb * S * 64;
      const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * 64;
      float* dq_base = a.dqkv + static_cast<int64_t>(b) * S * row_stride + h * 64;
      // DETERMINISM: dQ = (((p0 + p1) + p2) + ...) * scale over the key blocks holding a key <=
      // the row (causal) or all of them.
      for (int idx = tid; idx < S * 16; idx += NT) {
        const int i = idx >> 4, c4 = idx & 15;
        const int last = CAUSAL ? min(nkb - 1, i / KB) : nkb - 1;
        float4 v = __ldcg(reinterpret_cast<const float4*>(part + static_cast<int64_t>(i) * 64) + c4);
        for (int j = 1; j <= last; ++j) {
          const float4 p = __ldcg(
              reinterpret_cast<const float4*>(part + (static_cast<int64_t>(j) * S + i) * 64) + c4);
          v = make_float4(v.x + p.x, v.y + p.y, v.z + p.z, v.w + p.w);
        }
        reinterpret_cast<float4*>(dq_base + i * row_stride)[c4] =
            make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (w == 0) tc::tmem_dealloc(tbase, TMEM_COLS);
}

}  // namespace

cudaError_t setup_bwd_tc_attributes() {
  cudaError_t e = cudaFuncSetAttribute(bwd_tc_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(bwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              SMEM_ALLOC);
}

cudaError_t launch_bwd_tc(const BwdArgs& args, int causal, cudaStream_t stream) {
  BwdArgs a = args;
  a.n_kblocks = (a.S + KB - 1) / KB;
  const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(a.n_kblocks) * a.B * a.H));
  if (causal) return launch_pdl(bwd_tc_kernel<true>, grid, dim3(NT), SMEM_ALLOC, stream, a);
  return launch_pdl(bwd_tc_kernel<false>, grid, dim3(NT), SMEM_ALLOC, stream, a);
}

}  // namespace cfa
