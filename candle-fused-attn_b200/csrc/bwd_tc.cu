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
// Block: 16 compute warps and one MMA warp own a key block of KB = 128 keys of one (batch, head)
// and walk its query tiles of QT = 64. Compute thread (warp w < 16, lane l) owns key row
// 32 (w % 4) + l -- its TMEM lane -- and the 16 columns of group w / 4; warp 16 issues every MMA.
// Per query tile n:
//   T1:  S^T  = K Q^T      A: K parts (shared, K-major)   B: Q parts (K-major)        -> TMEM S
//        dP^T = V dO^T     A: V parts (TMEM, loaded once)  B: dO parts                -> TMEM DP
//   C1a: (during dP^T) the threads form P^T = exp(S^T * scale - L) (masked) and put its parts
//        into TMEM (the A operand of dV), over the S^T columns each has just read and in T_X;
//   C1b: (during dV) dS^T = P^T o (dP^T - D), its parts into shared memory;
//   T2:  dV  += P^T dO     A: P^T parts (TMEM)             B: dO parts read MN-major  -> TMEM DV
//        dK  += dS^T Q     A: dS^T parts (K-major)         B: Q parts read MN-major   -> TMEM DK
//        dQ_t = dS K       A: dS^T parts read MN-major (M = 64 queries)  B: K parts read MN-major,
//                          keys 0-63 and 64-127 in two windows                    -> TMEM DQ0, DQ1
//   C3:  (during T2) the next tile's Q, dO into their parts -- two buffers, by tile parity;
//   C2:  (during T1 of the next tile) dV, dK fold into fp32 registers; the tile's dQ partial goes
//        to the workspace.
// The hand-offs are mbarriers: S^T, dP^T, dV and dK + dQ commit one by one; the compute warps
// arrive (one per warp) when P^T's parts, dS^T's parts and the next tile's Q, dO parts are in
// place. The MMA warp issues T1(n + 1) once dV(n) has completed (it reads P^T(n) from the columns
// S^T(n + 1) writes), queued behind dK(n), dQ(n). The block that finishes last for its (batch,
// head) sums the dQ partials in key-block order (the no-wait path of bwd_ffma.cu: bit-identical
// for every schedule).
// S^T takes its six products in the forward kernel's order (A and B swapped), so the scores match
// fwd_tc.cu's and the recomputed P matches the forward's L.
//
// Split tail. With one block per SM, a grid of U key blocks runs in waves of P (the SM count); the
// R = U mod P key blocks of the partial last wave would hold R SMs for a whole block's time while
// the others idle. On the no-wait path (non-causal), the launcher runs each of them as k blocks
// (k = min(query tiles, P / R)), part p taking the p-th contiguous range of query tiles: the
// helpers (p >= 1) store each tile's dV, dK TMEM windows -- the values one block would fold --
// in workspace space the 128-key blocks leave unused, and raise a flag; the first part folds its
// own tiles, then the helpers' windows in tile order, so dV, dK are the one-block sums bit for
// bit, and only it writes dV, dK and counts the key block in. The roles go by a ticket drawn at
// the block's start, helpers first, and the helpers never wait on anyone, so a running first
// part's bounded wait always ends.
//
// Every mbarrier wait is bounded; an expired wait sets the workspace error flag
// (cfa_bwd_status reads it) and the block writes nothing.
#include <cuda_bf16.h>

#include "cfa_common.cuh"
#include "cfa_internal.h"
#include "cfa_split.cuh"
#include "cfa_tc.cuh"

namespace cfa {
using tc::kmaj_off;
using tc::split16;
using tc::split8;
using tc::store_parts;
using tc::tmem_ld8;
using tc::tmem_st8;
namespace {

constexpr int KB = 128;   // keys per block: MMA M of S^T, dP^T, dV, dK
constexpr int QT = 64;    // queries per tile: MMA N of S^T, dP^T; M of dQ
constexpr int NT = 512;   // compute threads (16 warps)
constexpr int NB = NT + 32;  // and the MMA warp
constexpr int PART_K = KB * 64 * 2;  // one bf16 part of a [128][64] operand
constexpr int PART_Q = QT * 64 * 2;  // one bf16 part of a [64][64] operand
constexpr int OFF_K = 0;                      // K parts [128 keys][64 d]
constexpr int OFF_Q = OFF_K + 3 * PART_K;     // Q parts [64 q][64 d], two tiles
constexpr int OFF_DO = OFF_Q + 6 * PART_Q;    // dO parts [64 q][64 d], two tiles
constexpr int OFF_DS = OFF_DO + 6 * PART_Q;   // dS^T parts [128 keys][64 q] (first: K staged)
constexpr int OFF_ST = OFF_DS + 3 * PART_K;   // staging: the next tile's Q, dO (fp32)
constexpr int OFF_LD = OFF_ST + 2 * QT * 64 * 4;  // L, D of two tiles: float [2][2][64]
constexpr int OFF_BAR = OFF_LD + 2 * 2 * QT * 4;  // eight mbarriers, the TMEM base, four ints
constexpr int SMEM = OFF_BAR + 96;
constexpr int SMEM_ALLOC = SMEM + 1024;
static_assert(SMEM_ALLOC <= 232448, "shared memory per block");
// TMEM columns (lane = key row). V's parts, the A operand of dP^T: part i, K-step ks (16 dims) in
// the 8 columns T_V + 32 i + 8 ks. S^T, dP^T of the current tile; P^T's parts (the A operand of
// dV: pt_col) over the S^T columns each thread has read and in T_X; dV, dK; dQ's two 64-key
// windows (M = 64).
constexpr uint32_t T_V = 0, T_S = 96, T_DP = 160, T_DV = 224, T_DK = 288, T_DQ0 = 352,
                   T_DQ1 = 416, T_X = 480;
constexpr uint32_t TMEM_COLS = 512;

// A split tail's window of one query tile (dV, dK sums of the tile as TMEM holds them, before the
// fold): WIN floats as float4 items [which: dV, dK][c4][column group][key row], so a warp's 32
// rows of one item are 512 contiguous bytes (coalesced stores, conflict-free shared-memory reads).
template <int HD>
struct TailWindow {
  static constexpr int WIN = 2 * KB * HD;
  static constexpr int CG = HD / 16;  // column groups of 16 floats
  __host__ __device__ static constexpr int item(int which, int c4, int cg, int row) {
    return ((which * 4 + c4) * CG + cg) * KB + row;
  }
};

// P^T part i of K-step ks (queries 16 ks .. 16 ks + 15: the columns of group ks): parts 0, 1 over
// that group's S^T columns, part 2 in T_X + 8 ks -- dP^T stays whole until dS^T is formed from
// it, while dV already runs.
__host__ __device__ constexpr uint32_t pt_col(int i, int ks) {
  return i < 2 ? T_S + 16 * ks + 8 * i : T_X + 8 * ks;
}
static_assert(T_X + 32 == TMEM_COLS, "TMEM budget");

// Row items (row r, elements 8 kc .. 8 kc + 7): item c takes row 8 (c / 64) + c % 8 and chunk
// (c / 8) % 8 (a quarter-warp writes 8 rows of one chunk: 8 bank groups). Every thread copies
// (cp.async) the fp32 chunks it splits into slots of its own: slot j of thread t at
// (j * NT + t) * 16 bytes.
__device__ __forceinline__ void row_item(int c, int& r, int& kc) {
  r = 8 * (c >> 6) + (c & 7);
  kc = (c >> 3) & 7;
}

// (Head dim 32: the row's chunks past the head dim are zero-filled, so the parts are those of a
// 64-wide row whose upper half is zero.)
template <int HD>
__device__ __forceinline__ void stage_row_item(unsigned char* st, int slot, int c, const float* src,
                                               int64_t stride, int r0, int seq) {
  int r, kc;
  row_item(c, r, kc);
  const bool ok = r0 + r < seq && 8 * kc < HD;
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

// Row item c of a row-major staging area with rows of 68 floats (rows >= valid and columns >= HD
// read as zeros) into the K-major parts at part_bytes apart.
template <int HD>
__device__ __forceinline__ void split_staged_row(unsigned char* parts, int part_bytes,
                                                 const float* rows, int c, int valid) {
  int r, kc;
  row_item(c, r, kc);
  float x[8];
  if (r < valid && 8 * kc < HD) {
    const float4 u = reinterpret_cast<const float4*>(rows + r * 68 + 8 * kc)[0];
    const float4 v = reinterpret_cast<const float4*>(rows + r * 68 + 8 * kc)[1];
    x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = v.x, x[5] = v.y, x[6] = v.z, x[7] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.0f;
  }
  store_parts(parts, part_bytes, kmaj_off(r, kc), x);
}

// One window: six split products over STEPS K-steps into the fresh accumulator `d`; descriptors
// advance by A_STEP / B_STEP bytes per step and by A_PART / B_PART bytes per part. Part pairs
// (P0(p), P1(p)) -- the small (0, 1), (1, 0), (0, 2), (1, 1), (2, 0) of every step, then the
// (0, 0) of every step -- or, SWAP, (P1(p), P0(p)): the order in which the forward forms its
// products when A and B trade places. Called by the whole MMA warp (tc::mma_bf16_warp).
__host__ __device__ constexpr int P0(int p) { return p == 2 || p == 4 ? 1 : (p == 5 ? 2 : 0); }
__host__ __device__ constexpr int P1(int p) { return p == 1 || p == 4 ? 1 : (p == 3 ? 2 : 0); }
template <int STEPS, int A_PART, int B_PART, int A_STEP, int B_STEP, bool SWAP>
__device__ __forceinline__ void issue6(uint32_t d, tc::Desc ad, tc::Desc bd, uint32_t idesc) {
  const uint32_t alo = tc::opaque(ad.lo), blo = tc::opaque(bd.lo);
#pragma unroll
  for (int ks = 0; ks < STEPS; ++ks)
#pragma unroll
    for (int p = 1; p < 6; ++p) {
      const int pa = SWAP ? P1(p) : P0(p), pb = SWAP ? P0(p) : P1(p);
      tc::mma_bf16_warp(d, alo + ((pa * A_PART + A_STEP * ks) >> 4), ad.hi,
                        blo + ((pb * B_PART + B_STEP * ks) >> 4), bd.hi, idesc, ks > 0 || p > 1);
    }
#pragma unroll
  for (int ks = 0; ks < STEPS; ++ks)
    tc::mma_bf16_warp(d, alo + ((A_STEP * ks) >> 4), ad.hi, blo + ((B_STEP * ks) >> 4), bd.hi,
                      idesc, 1);
}

// The same window with the A operand in TMEM: part i of K-step ks at column acol(i, ks).
template <int B_PART, int B_STEP, typename ACol, int STEPS = 4>
__device__ __forceinline__ void issue6_tmem_a(uint32_t d, ACol acol, tc::Desc bd, uint32_t idesc) {
  const uint32_t blo = tc::opaque(bd.lo);
#pragma unroll
  for (int ks = 0; ks < STEPS; ++ks)
#pragma unroll
    for (int p = 1; p < 6; ++p)
      tc::mma_bf16_tmem_a_warp(d, acol(P0(p), ks), blo + ((P1(p) * B_PART + B_STEP * ks) >> 4),
                               bd.hi, idesc, ks > 0 || p > 1);
#pragma unroll
  for (int ks = 0; ks < STEPS; ++ks)
    tc::mma_bf16_tmem_a_warp(d, acol(0, ks), blo + ((B_STEP * ks) >> 4), bd.hi, idesc, 1);
}

constexpr float LOG2E = 1.4426950408889634f;  // log2(e), rounded to fp32

// Packed fp32 pairs (tc::pack2 / unpack2), one instruction a pair.
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2v(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Eight floats to global memory in one 32-byte store (address 32-byte aligned), cached in L2 only.
__device__ __forceinline__ void st_cg_v8(float* p, const float (&v)[8]) {
  asm volatile("st.global.cg.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]),
               "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

// atomicAdd with acquire-release semantics at GPU scope.
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Named barrier 1: the 16 compute warps (the MMA warp never takes part).
__device__ __forceinline__ void bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <bool CAUSAL, int HD>
__global__ void __launch_bounds__(NB, 1) bwd_tc_kernel(const BwdArgs a) {
  static_assert(HD == 64 || HD == 32, "head dims of the tensor-core backward");
  constexpr int KSD = HD / 16;  // K-steps of the products that reduce over the head dim
  constexpr int WIN = TailWindow<HD>::WIN;
  constexpr auto win4 = TailWindow<HD>::item;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* Kp = sm + OFF_K;
  unsigned char* Qp = sm + OFF_Q;
  unsigned char* dOp = sm + OFF_DO;
  unsigned char* dSp = sm + OFF_DS;
  unsigned char* st = sm + OFF_ST;
  float* ld = reinterpret_cast<float*>(sm + OFF_LD);  // [buf][0: L, 1: D][64]
  // Commits (each covers every earlier MMA of the block) and arrivals (one per compute warp).
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + OFF_BAR);  // S^T of a tile done
  uint64_t* bar_t2 = bar_s + 1;  // dK, dQ of a tile done: every MMA of the tile
  uint64_t* bar_c1 = bar_s + 2;  // dS^T of a tile in shared memory (arrivals)
  uint64_t* bar_q = bar_s + 3;   // Q, dO parts of the next tile in place (arrivals)
  uint64_t* bar_ld = bar_s + 4;  // bulk copies: the prologue's rows, then the tail's windows
  uint64_t* bar_dp = bar_s + 5;  // dP^T of a tile done
  uint64_t* bar_p = bar_s + 6;   // P^T's parts of a tile in TMEM (arrivals)
  uint64_t* bar_dv = bar_s + 7;  // dV of a tile done
  uint32_t* tbase_p = reinterpret_cast<uint32_t*>(bar_s + 8);
  int* s_int = reinterpret_cast<int*>(bar_s + 9);

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const bool mma_warp = w == NT / 32;   // warp 16 issues every MMA
  const int row = 32 * (w & 3) + lane;  // key row: TMEM lane (compute warps)
  const int cg = (w >> 2) & 3;          // column group: 16 queries (S, dP) or dims (dV, dK, dQ)
  const int S = a.S;
  const int nkb = a.n_kblocks;
  const int BH = a.B * a.H;
  // The work item. With the dQ partials (no-wait path): the block index, (b, h)-major, so a
  // (b, h)'s key blocks run side by side and its last one finishes early. With the turn chain: a
  // ticket drawn after the prep kernel's wait, key-block-major -- a block waits only on key block
  // kb - 1 of its (b, h), which holds a smaller ticket, so it is running or done.
  const bool chain = a.dq_part == nullptr;
  int ticket = static_cast<int>(blockIdx.x);
  if (chain) {
    if (tid == 0) {
      griddep_wait();  // the cleared ticket and counters
      s_int[1] = atomicAdd(a.ticket, 1);
    }
    __syncthreads();
    ticket = s_int[1];
  }
  // Split tail (no-wait path): the key blocks from a.tail_base on -- the grid's last partial wave
  // -- run as a.tail_parts blocks each, part p taking the p-th contiguous range of the query tiles.
  // The helpers (parts >= 1) leave their tiles' dV, dK windows in a.tail_win; the first part adds
  // them after its own, in tile order: the same sums as one block, bit for bit. Only the first
  // part writes dV, dK and counts the key block in. The roles go by a ticket drawn at the start,
  // helpers first, so a first part that runs finds every helper running or done (no assumption
  // on the order in which the hardware starts blocks): its wait always ends.
  int part = 0, nparts = 1, tail_r = 0;
  if (!CAUSAL && !chain && a.tail_parts > 1 && ticket >= a.tail_base) {
    if (tid == 0) {
      griddep_wait();  // the tail's ticket counter, cleared by the prep kernel
      s_int[1] = atomicAdd(a.tail_flag + a.tail_units * a.tail_parts, 1);
    }
    __syncthreads();
    const int j = s_int[1];
    const int g = j / a.tail_units;
    tail_r = j - g * a.tail_units;
    nparts = a.tail_parts;
    part = g + 1 < nparts ? g + 1 : 0;
    ticket = a.tail_base + tail_r;
  }
  const int kb = chain ? ticket / BH : ticket % nkb;
  const int bh = chain ? ticket % BH : ticket / nkb;
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kb * KB;
  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* kp = a.k + b * a.k_sb + h * a.k_sh;
  const float* vp = a.v + b * a.v_sb + h * a.v_sh;
  const float* gp = a.d_o + b * a.do_sb + h * a.do_sh;
  const float* lp = a.lse + static_cast<int64_t>(bh) * S;
  const float* dp = a.dsum + static_cast<int64_t>(bh) * S;
  const int t_first = CAUSAL ? k0 / QT : 0;  // queries before the block's first key see none
  const int n_all = (S + QT - 1) / QT - t_first;  // the key block's query tiles, >= 1 (k0 < S)
  const int n_lo = part * n_all / nparts, n_hi = (part + 1) * n_all / nparts;
  const int t_begin = t_first + n_lo;  // this block's first query tile
  int* turn = a.turn + static_cast<int64_t>(bh) * a.n_qtiles;  // turn chain: per 64-query tile
  const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * HD;  // dqkv floats per (b, s)
  float* dq_base = a.dqkv + static_cast<int64_t>(b) * S * row_stride + h * HD;
  const int N = n_hi - n_lo;  // this block's query tiles, >= 1 (a.tail_parts <= n_all)
  bool err0 = false;

  if (tid == 0) {
    tc::mbar_init(bar_s, 1);
    tc::mbar_init(bar_t2, 1);
    tc::mbar_init(bar_c1, NT / 32);
    tc::mbar_init(bar_q, NT / 32);
    tc::mbar_init(bar_ld, 1);
    tc::mbar_init(bar_dp, 1);
    tc::mbar_init(bar_p, NT / 32);
    tc::mbar_init(bar_dv, 1);
    tc::fence_mbar_init();
    tc::mbar_arrive_expect_tx(bar_ld, 4u * HD * (2 * min(KB, S - k0) + 2 * min(QT, S - t_begin * QT)));
  }
  griddep_launch_dependents();

  // Q, dO of tile n into this thread's staging slots (Q: slots 0-1, dO: 2-3) and its L, D into
  // L / D buffer n % 2 (threads 0-127).
  auto stage_ld = [&](int n) {
    if (tid < 2 * QT) {
      const int r = tid & 63, i = (t_begin + n) * QT + r;
      const bool ok = i < S;
      cp_async4(ld + (n & 1) * 128 + (tid < QT ? 0 : QT) + r, (tid < QT ? lp : dp) + (ok ? i : 0),
                ok ? 4 : 0);
    }
  };
  auto stage_tile = [&](int n) {
    const int q0 = (t_begin + n) * QT;
    stage_row_item<HD>(st, 0, tid, qp, a.q_ss, q0, S);
    stage_row_item<HD>(st, 1, tid, gp, a.do_ss, q0, S);
    stage_ld(n);
  };
  // The block one wave later (work item + a.wave_ctas) starts by reading its key block's K, V rows
  // and its first query tile's Q, dO rows, all at once across the wave: pull them into L2 while
  // this wave computes and HBM is otherwise idle (one 256-byte row per thread).
  auto prefetch_next_wave = [&]() {
    const int nb = ticket + a.wave_ctas;
    if (a.wave_ctas <= 0 || nparts > 1 || nb >= nkb * BH || tid >= 2 * KB + 2 * QT) return;
    const int nkb2 = chain ? nb / BH : nb % nkb, nbh = chain ? nb % BH : nb / nkb;
    const int nb_b = nbh / a.H, nb_h = nbh % a.H;
    const int r = tid < 2 * KB ? (tid & (KB - 1)) : (tid & (QT - 1));
    const int row = tid < 2 * KB ? nkb2 * KB + r : (CAUSAL ? nkb2 * KB : 0) + r;
    if (row >= S) return;
    const float* src;
    if (tid < KB) src = a.k + nb_b * a.k_sb + nb_h * a.k_sh + static_cast<int64_t>(row) * a.k_ss;
    else if (tid < 2 * KB) src = a.v + nb_b * a.v_sb + nb_h * a.v_sh + static_cast<int64_t>(row) * a.v_ss;
    else if (tid < 2 * KB + QT) src = a.q + nb_b * a.q_sb + nb_h * a.q_sh + static_cast<int64_t>(row) * a.q_ss;
    else src = a.d_o + nb_b * a.do_sb + nb_h * a.do_sh + static_cast<int64_t>(row) * a.do_ss;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "n"(4 * HD) : "memory");
  };
  auto split_tile = [&](int n) {
    split_row_item(Qp + (n & 1) * 3 * PART_Q, PART_Q, st, 0, tid);
    split_row_item(dOp + (n & 1) * 3 * PART_Q, PART_Q, st, 1, tid);
  };

  // Prologue: K's parts into shared memory, V's into TMEM (this thread's key row and 16 dims:
  // K-step cg of the A operand of dP^T), tile 0's Q and dO parts. The rows of K, V, Q, dO travel
  // as one bulk copy each (threads 0-383, one row apiece) into row-major staging with rows of
  // LDP = 68 floats (the dS^T and staging buffers: K, V; the second Q and dO part buffers: Q, dO
  // of tile 0); rows past the sequence are not copied and read as zeros. L, D and the cleared
  // counters come after the prep kernel's wait.
  constexpr int LDP = 68;
  float* k_rows = reinterpret_cast<float*>(dSp);
  float* v_rows = k_rows + KB * LDP;
  float* q_rows = reinterpret_cast<float*>(Qp + 3 * PART_Q);
  float* o_rows = reinterpret_cast<float*>(dOp + 3 * PART_Q);
  static_assert(2 * KB * LDP * 4 <= 3 * PART_K + 2 * QT * 64 * 4 && QT * LDP * 4 <= 3 * PART_Q,
                "prologue staging");
  const int nk = min(KB, S - k0), nq = min(QT, S - t_begin * QT);
  __syncthreads();  // the mbarriers' initialisation
  if (mma_warp) {  // TMEM, by the warp that is idle while the rows travel (it also frees it)
    tc::tmem_alloc(tbase_p, TMEM_COLS);
    tc::tmem_relinquish();
  }
  float vx[16];
  if (!mma_warp) {
    if (tid < 2 * KB + 2 * QT) {
      const int r = tid < 2 * KB ? (tid & (KB - 1)) : (tid & (QT - 1));
      if (tid < KB) {
        if (r < nk) tc::bulk_load(k_rows + r * LDP, kp + static_cast<int64_t>(k0 + r) * a.k_ss, 4 * HD, bar_ld);
      } else if (tid < 2 * KB) {
        if (r < nk) tc::bulk_load(v_rows + r * LDP, vp + static_cast<int64_t>(k0 + r) * a.v_ss, 4 * HD, bar_ld);
      } else if (tid < 2 * KB + QT) {
        if (r < nq)
          tc::bulk_load(q_rows + r * LDP, qp + static_cast<int64_t>(t_begin * QT + r) * a.q_ss, 4 * HD, bar_ld);
      } else if (r < nq) {
        tc::bulk_load(o_rows + r * LDP, gp + static_cast<int64_t>(t_begin * QT + r) * a.do_ss, 4 * HD, bar_ld);
      }
    }
    griddep_wait();  // L, D, the cleared counters: the prep kernel's writes
    stage_ld(0);
    cp_async_commit();
    err0 = !tc::mbar_wait(bar_ld, 0, WAIT_TIMEOUT_NS);
    cp_async_wait_all();
    split_staged_row<HD>(Kp, PART_K, k_rows, tid, nk);
    split_staged_row<HD>(Kp, PART_K, k_rows, tid + NT, nk);
    split_staged_row<HD>(Qp, PART_Q, q_rows, tid, nq);
    split_staged_row<HD>(dOp, PART_Q, o_rows, tid, nq);
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      const float4 u = row < nk && 16 * cg < HD
                           ? reinterpret_cast<const float4*>(v_rows + row * LDP + 16 * cg)[c4]
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      vx[4 * c4] = u.x;
      vx[4 * c4 + 1] = u.y;
      vx[4 * c4 + 2] = u.z;
      vx[4 * c4 + 3] = u.w;
    }
    tc::fence_async_smem();
  }
  tc::fence_before_sync();
  __syncthreads();  // the TMEM base; L, D of tile 0 (threads 0-127); the K staging read
  tc::fence_after_sync();
  const uint32_t tbase = *tbase_p;
  const uint32_t lane_sel = static_cast<uint32_t>(32 * (w & 3)) << 16;
  if (!mma_warp) {
    uint32_t vparts[3][8];
    split16(vx, vparts);
#pragma unroll
    for (int i = 0; i < 3; ++i) tmem_st8(tbase + lane_sel + T_V + 32 * i + 8 * cg, vparts[i]);
    tc::tmem_wait_st();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  bool err = err0;
  uint32_t ld_phase = 1;  // bar_ld's next phase: the prologue's copies completed phase 0
  const int key = k0 + row;
  const uint64_t nsc2 = tc::pack2(-a.scale, -a.scale);     // L - s scale = fma(s, -scale, L)
  const uint64_t nl2e2 = tc::pack2(-LOG2E, -LOG2E);        // e^-y = 2^(-y log2 e)
  float dv[16], dk[16];  // compute threads: dV, dK of the key row, this thread's 16 dims
#pragma unroll
  for (int c = 0; c < 16; ++c) dv[c] = dk[c] = 0.0f;
  if (mma_warp) {
    {  // every lane runs the loop (warp-uniform); one elected lane issues each MMA and commit
      const uint32_t id128 = tc::idesc_f32acc(1, KB, QT);           // S^T, dP^T: M 128, N 64
      const uint32_t id_mn = tc::idesc_f32acc(1, KB, HD) | (1u << 16);  // dV, dK: N = d, B MN
      const uint32_t id_dq = tc::idesc_f32acc(1, QT, HD) | (1u << 15) | (1u << 16);  // M 64
      const uint32_t sK = tc::smem_u32(Kp), sS = tc::smem_u32(dSp);
      // S^T (the forward's product order) and dP^T (A: V's parts in TMEM) of tile n, committed
      // one by one: the compute warps form P^T while dP^T runs.
      auto issue_t1 = [&](int n) {
        const uint32_t sQ = tc::smem_u32(Qp + (n & 1) * 3 * PART_Q);
        const uint32_t sO = tc::smem_u32(dOp + (n & 1) * 3 * PART_Q);
        issue6<KSD, PART_K, PART_Q, 256, 256, true>(tbase + T_S,
                                                  tc::split_desc(tc::desc_kmajor(sK, 128, 1024)),
                                                  tc::split_desc(tc::desc_kmajor(sQ, 128, 1024)), id128);
        tc::commit_warp(bar_s);
        auto vcol = [&](int i, int ks) { return tbase + T_V + 32 * i + 8 * ks; };
        issue6_tmem_a<PART_Q, 256, decltype(vcol), KSD>(
            tbase + T_DP, vcol, tc::split_desc(tc::desc_kmajor(sO, 128, 1024)), id128);
        tc::commit_warp(bar_dp);
      };
      // dV (A: P^T's parts in TMEM) of tile n: it runs while the compute warps form dS^T.
      auto issue_dv = [&](int n) {
        const uint32_t sO = tc::smem_u32(dOp + (n & 1) * 3 * PART_Q);
        issue6_tmem_a<PART_Q, 2048>(tbase + T_DV, [&](int i, int ks) { return tbase + pt_col(i, ks); },
                                    tc::split_desc(tc::desc_kmajor(sO, 1024, 128)), id_mn);
        tc::commit_warp(bar_dv);
      };
      // dK, dQ (two windows of 64 keys) of tile n.
      auto issue_t2 = [&](int n) {
        const uint32_t sQ = tc::smem_u32(Qp + (n & 1) * 3 * PART_Q);
        issue6<4, PART_K, PART_Q, 256, 2048, false>(tbase + T_DK,
                                                    tc::split_desc(tc::desc_kmajor(sS, 128, 1024)),
                                                    tc::split_desc(tc::desc_kmajor(sQ, 1024, 128)), id_mn);
        const tc::Desc as_mn = tc::split_desc(tc::desc_kmajor(sS, 1024, 128));
        const tc::Desc bk_mn = tc::split_desc(tc::desc_kmajor(sK, 1024, 128));
        issue6<4, PART_K, PART_K, 2048, 2048, false>(tbase + T_DQ0, as_mn, bk_mn, id_dq);
        issue6<4, PART_K, PART_K, 2048, 2048, false>(
            tbase + T_DQ1, {as_mn.lo + (8192 >> 4), as_mn.hi}, {bk_mn.lo + (8192 >> 4), bk_mn.hi},
            id_dq);
        tc::commit_warp(bar_t2);
      };
      // The tensor core's order: S^T(n), dP^T(n), dV(n) once P^T(n) is in TMEM, dK(n), dQ(n)
      // once dS^T(n) is in shared memory, then S^T(n + 1) -- over P^T(n)'s columns, once dV(n) has
      // completed -- and dP^T(n + 1), queued behind dK(n), dQ(n).
      issue_t1(0);
      for (int n = 0; n < N; ++n) {
        err |= !tc::mbar_wait(bar_p, n & 1, WAIT_TIMEOUT_NS);
        tc::fence_after_sync();
        issue_dv(n);
        err |= !tc::mbar_wait(bar_c1, n & 1, WAIT_TIMEOUT_NS);  // dP^T(n) read, dS^T(n) stored
        tc::fence_after_sync();
        issue_t2(n);
        if (n + 1 < N) {
          err |= !tc::mbar_wait(bar_q, n & 1, WAIT_TIMEOUT_NS);
          err |= !tc::mbar_wait(bar_dv, n & 1, WAIT_TIMEOUT_NS);  // dV(n) has read P^T(n)
          tc::fence_after_sync();
          issue_t1(n + 1);
        }
      }
    }
  } else {
    if (N > 1) stage_tile(1);  // while the MMA warp issues T1(0)
    cp_async_commit();
    for (int n = 0; n < N; ++n) {
      const int q0 = (t_begin + n) * QT;
      // (C1a) P^T for this thread's 16 queries, its parts into TMEM (pt_col) for dV -- while the
      // tensor core computes dP^T.
      err |= !tc::mbar_wait(bar_s, n & 1, WAIT_TIMEOUT_NS);
      tc::fence_after_sync();
      const float* Lt = ld + (n & 1) * 128;
      const float* Dt = Lt + QT;
      const bool edge = (q0 + QT > S) || (k0 + KB > S) || (CAUSAL && k0 + KB - 1 > q0);
      float pr[16];
      tc::tmem_ld16(tbase + lane_sel + T_S + 16 * cg, pr);
      tc::tmem_wait_ld();
      // Two halves of 8 queries, each half's parts stored (columns 4 h .. 4 h + 3 of its K-step)
      // while the next half is formed: the stores' latency no longer trails the arithmetic.
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int u = 8 * hh; u < 8 * hh + 8; u += 2) {
          const int ql = 16 * cg + u;
          // P = e^(s * scale - L): the argument with one rounding (L - s scale by one fma, so the
          // cancellation is exact), then 2^(arg log2 e) on the SFU (ex2.approx, max relative
          // error about 2^-22). Pairs of queries in packed fp32.
          const uint64_t l2 = *reinterpret_cast<const uint64_t*>(Lt + ql);
          float x0, x1;
          tc::unpack2(mul2(fma2v(tc::pack2(pr[u], pr[u + 1]), nsc2, l2), nl2e2), x0, x1);
          float p0 = ex2(x0), p1 = ex2(x1);
          if (edge) {
            if (!(q0 + ql < S && key < S && !(CAUSAL && key > q0 + ql))) p0 = 0.0f;
            if (!(q0 + ql + 1 < S && key < S && !(CAUSAL && key > q0 + ql + 1))) p1 = 0.0f;
          }
          pr[u] = p0;
          pr[u + 1] = p1;
        }
        const float xh[8] = {pr[8 * hh], pr[8 * hh + 1], pr[8 * hh + 2], pr[8 * hh + 3],
                             pr[8 * hh + 4], pr[8 * hh + 5], pr[8 * hh + 6], pr[8 * hh + 7]};
        uint4 h0, h1, h2;
        split8(xh, h0, h1, h2);
        tc::tmem_st4(tbase + lane_sel + pt_col(0, cg) + 4 * hh, h0);
        tc::tmem_st4(tbase + lane_sel + pt_col(1, cg) + 4 * hh, h1);
        tc::tmem_st4(tbase + lane_sel + pt_col(2, cg) + 4 * hh, h2);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_p);
      // (C1b) dS^T = P^T o (dP^T - D), its parts into shared memory for dK, dQ -- while the tensor
      // core computes dV.
      err |= !tc::mbar_wait(bar_dp, n & 1, WAIT_TIMEOUT_NS);
      tc::fence_after_sync();
#pragma unroll
      for (int h8 = 0; h8 < 2; ++h8) {
        const uint32_t col = 16 * cg + 8 * h8;
        float gb[8];
        tmem_ld8(tbase + lane_sel + T_DP + col, gb);
        tc::tmem_wait_ld();
        float ds[8];
#pragma unroll
        for (int u = 0; u < 8; u += 2) {
          const uint64_t d2 = *reinterpret_cast<const uint64_t*>(Dt + col + u);
          tc::unpack2(mul2(tc::pack2(pr[8 * h8 + u], pr[8 * h8 + u + 1]),
                           tc::sub2(tc::pack2(gb[u], gb[u + 1]), d2)),
                      ds[u], ds[u + 1]);
        }
        store_parts(dSp, PART_K, kmaj_off(row, 2 * cg + h8), ds);
      }
      tc::fence_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_c1);
      if (n == 0) prefetch_next_wave();
      // (C3) The next tile's Q, dO into their parts (its buffer was last read by T2(n - 1)), while
      // the tensor core computes dV, dK, dQ; the tile after it travels.
      if (n + 1 < N) {
        cp_async_wait_all();
        bar_sync(1, NT);  // L, D of tile n + 1 in place; every thread is past C1(n)
        split_tile(n + 1);
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_q);
        if (n + 2 < N) stage_tile(n + 2);
        cp_async_commit();
      }
      // (C2) Fold dV, dK; write the dQ partial.
      err |= !tc::mbar_wait(bar_t2, n & 1, WAIT_TIMEOUT_NS);
      tc::fence_after_sync();
      float xb[16], xs[16];
      tc::tmem_ld16(tbase + lane_sel + T_DV + 16 * cg, xb);
      tc::tmem_ld16(tbase + lane_sel + T_DK + 16 * cg, xs);
      tc::tmem_wait_ld();
      if (16 * cg < HD) {  // dV, dK have HD columns
        if (part == 0) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            dv[c] += xb[c];
            dk[c] += xs[c];
          }
        } else {  // a split tail's helper: the tile's windows for the first part (win4)
          float4* wv = reinterpret_cast<float4*>(a.tail_win) +
                       (static_cast<int64_t>(tail_r) * n_all + n_lo + n) * (WIN / 4);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            __stcg(wv + win4(0, c4, cg, row),
                   make_float4(xb[4 * c4], xb[4 * c4 + 1], xb[4 * c4 + 2], xb[4 * c4 + 3]));
            __stcg(wv + win4(1, c4, cg, row),
                   make_float4(xs[4 * c4], xs[4 * c4 + 1], xs[4 * c4 + 2], xs[4 * c4 + 3]));
          }
        }
      }
      // dQ (M = 64): query row 16 (w % 4) + lane in lanes 0-15 of each quarter; the two windows.
      tc::tmem_ld16(tbase + lane_sel + T_DQ0 + 16 * cg, xb);
      tc::tmem_ld16(tbase + lane_sel + T_DQ1 + 16 * cg, xs);
      tc::tmem_wait_ld();
      const int qi = q0 + 16 * (w & 3) + lane;
      if (!chain) {
        if (lane < 16 && qi < S && 16 * cg < HD && !err) {
          // Two 32-byte stores: whole L2 sectors (16-byte stores 256 bytes apart across the warp
          // each wrote half of 16 sectors).
          float* dst = a.dq_part + ((static_cast<int64_t>(bh) * nkb + kb) * S + qi) * HD + 16 * cg;
#pragma unroll
          for (int c8 = 0; c8 < 2; ++c8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = xb[8 * c8 + u] + xs[8 * c8 + u];
            st_cg_v8(dst + 8 * c8, v);
          }
        }
      } else {
        // Turn chain: query tile t's contributors are key blocks 0 .. last (causal: those holding
        // a key <= the tile's last query); each adds its partial into dQ on its turn, through L2
        // (__ldcg / __stcg), and the last multiplies by `scale`: dQ = ((p0 + p1) + ...) * scale,
        // the no-wait path's sums bit for bit.
        const int t = t_begin + n;
        const int last = CAUSAL ? min(nkb - 1, min(S - 1, q0 + QT - 1) / KB) : nkb - 1;
        bool go = true;
        if (kb > 0) {
          if (tid == 0) {
            // (slot by tile parity: a thread may still read the last tile's flag)
            s_int[2 + (n & 1)] = wait_turn_bounded(turn + t, kb, a.err, a.timeout_ns, a.sink) ? 1 : 0;
            // ORDER: with the barrier below, extends thread 0's acquire to the compute warps.
            __threadfence();
          }
          bar_sync(1, NT);
          go = s_int[2 + (n & 1)] != 0;
        }
        if (go && lane < 16 && qi < S && 16 * cg < HD) {
          float4* dst = reinterpret_cast<float4*>(dq_base + qi * row_stride + 16 * cg);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            float4 v = make_float4(xb[4 * c4] + xs[4 * c4], xb[4 * c4 + 1] + xs[4 * c4 + 1],
                                   xb[4 * c4 + 2] + xs[4 * c4 + 2], xb[4 * c4 + 3] + xs[4 * c4 + 3]);
            if (kb > 0) {
              const float4 prev = __ldcg(dst + c4);
              v = make_float4(prev.x + v.x, prev.y + v.y, prev.z + v.z, prev.w + v.w);
            }
            if (kb == last) v = make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
            __stcg(dst + c4, v);
          }
        }
        err |= !go;
        if (kb < last) {
          // ORDER: every thread's dQ stores are visible GPU-wide before thread 0 hands the tile to
          // key block kb + 1 (its acquire in wait_turn_bounded).
          __threadfence();
          bar_sync(1, NT);
          if (tid == 0) st_release_gpu(turn + t, kb + 1);
        }
      }
    }
  }
  cp_async_wait_all();
  if (part == 0 && nparts > 1) {
    // The first part of a split key block: the helpers' tile windows, added after its own tiles'
    // in tile order (dv = ((w0 + w1) + w2) + ..., as one block folds them).
    if (tid == 0) {
      bool ok = true;
      for (int p = 1; p < nparts && ok; ++p)
        ok = wait_turn_bounded(a.tail_flag + tail_r * nparts + p, 1, a.err, a.timeout_ns, a.sink);
      s_int[2] = ok ? 1 : 0;
      // ORDER: with the barrier below, extends thread 0's acquires to the block (the windows and
      // the helpers' dQ partials; the count below passes the partials on to the summing block).
      __threadfence();
    }
    __syncthreads();
    const bool ok = s_int[2] != 0;
    err |= !ok;
    // The windows travel by bulk copy into shared memory (free since the last T2), up to WCH
    // tiles at a time: loads a thread issued itself would each wait out the L2 round trip.
    constexpr int WCH = OFF_BAR / (4 * WIN);
    static_assert(WCH >= 1, "one tile's windows fit in shared memory");
    const float4* wsm = reinterpret_cast<const float4*>(sm);
    for (int t0 = n_hi; ok && t0 < n_all; t0 += WCH) {
      const int nt = min(WCH, n_all - t0);
      if (tid == 0) {
        tc::fence_async_global();  // the windows the acquires made visible, for the copy engine
        tc::mbar_arrive_expect_tx(bar_ld, static_cast<uint32_t>(4 * WIN * nt));
        tc::bulk_load(sm, a.tail_win + (static_cast<int64_t>(tail_r) * n_all + t0) * WIN,
                      static_cast<uint32_t>(4 * WIN * nt), bar_ld);
      }
      const bool got = tc::mbar_wait(bar_ld, ld_phase & 1, WAIT_TIMEOUT_NS);
      ++ld_phase;
      err |= !got;
      if (got && !mma_warp && 16 * cg < HD) {
        for (int t = 0; t < nt; ++t) {
          const float4* wv = wsm + t * (WIN / 4);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            const float4 x = wv[win4(0, c4, cg, row)];
            const float4 y = wv[win4(1, c4, cg, row)];
            dv[4 * c4] += x.x, dv[4 * c4 + 1] += x.y, dv[4 * c4 + 2] += x.z, dv[4 * c4 + 3] += x.w;
            dk[4 * c4] += y.x, dk[4 * c4 + 1] += y.y, dk[4 * c4 + 2] += y.z, dk[4 * c4 + 3] += y.w;
          }
        }
      }
      // Every read of the chunk done before the next copy lands (and every thread leaves together).
      if (!__syncthreads_and(got)) break;
    }
  }
  err = __syncthreads_or(err);  // any expired wait in the block: nothing is written
  if (err) {
    if (tid == 0) flag_timeout(a.err, a.sink);
    tc::mbar_wait(bar_t2, (N - 1) & 1, WAIT_TIMEOUT_NS);  // no MMA left in flight
  } else if (part != 0) {
    // A helper of a split key block: its windows and dQ partials are written; hand them to the
    // first part (ORDER: every thread's stores are visible GPU-wide before thread 0's release).
    __threadfence();
    __syncthreads();
    if (tid == 0) st_release_gpu(a.tail_flag + tail_r * nparts + part, 1);
  } else {
    // The dQ partials' hand-off: after the barrier above, thread 0's acquire-release count
    // publishes every thread's partial stores (the barrier orders them before it) and, for the
    // last of the (b, h)'s key blocks, makes the other blocks' visible; that block sums them in
    // key-block order (the loads bypass L1).
    // dV into slot 2, dK * scale into slot 1 of dqkv [b, s, 3, h, 64] go through shared memory (the
    // dS^T and staging buffers, free since the last T2): rows of 68 floats (a 16-byte rotation per
    // row keeps both passes conflict-free), stored as whole rows at the end.
    constexpr int LDS = 68;
    float* sv = reinterpret_cast<float*>(dSp);
    float* sk = sv + KB * LDS;
    static_assert(2 * KB * LDS * 4 <= 3 * PART_K + 2 * QT * 64 * 4, "dV, dK rows fit");
    if (!mma_warp) {
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        reinterpret_cast<float4*>(sv + row * LDS + 16 * cg)[c4] =
            make_float4(dv[4 * c4], dv[4 * c4 + 1], dv[4 * c4 + 2], dv[4 * c4 + 3]);
        reinterpret_cast<float4*>(sk + row * LDS + 16 * cg)[c4] =
            make_float4(dk[4 * c4] * a.scale, dk[4 * c4 + 1] * a.scale, dk[4 * c4 + 2] * a.scale,
                        dk[4 * c4 + 3] * a.scale);
      }
    }
    __syncthreads();  // the dV, dK rows in place
    constexpr int C4 = HD / 4;  // float4 columns of a dQ, dK or dV row
    // Thread 0's count -- an acquire-release round trip through L2 -- travels while the block
    // stores the dV, dK rows.
    int count = -1;
    if (tid == 0 && !chain) count = atom_add_acq_rel(a.turn + bh, 1);
    // dV, dK rows out of shared memory: every 16 threads store one whole row.
    {
      const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * HD;
      for (int f = tid; f < 2 * KB * C4; f += NB) {
        const int which = f / (KB * C4), r = (f / C4) % KB, c4 = f % C4;
        if (k0 + r < S) {
          float* dst = a.dqkv + (static_cast<int64_t>(b) * S + k0 + r) * row_stride +
                       (2 - which) * a.H * HD + h * HD;
          reinterpret_cast<float4*>(dst)[c4] =
              reinterpret_cast<const float4*>((which ? sk : sv) + r * LDS)[c4];
        }
      }
    }
    if (tid == 0) s_int[0] = count;
    __syncthreads();
    const int64_t part_bytes = static_cast<int64_t>(nkb) * S * HD * 4;
    if (s_int[0] == nkb - 1 && part_bytes <= OFF_DS) {
      // The (b, h)'s partials, contiguous [nkb][S][64], as one bulk copy into shared memory (the
      // part buffers, free since the last T2; the dS^T buffer holds dV, dK), then summed there.
      const float* part = a.dq_part + static_cast<int64_t>(bh) * nkb * S * HD;
      const float* sp = reinterpret_cast<const float*>(sm);
      if (tid == 0) {
        tc::fence_async_global();  // the partials the count made visible, for the copy engine
        tc::mbar_arrive_expect_tx(bar_ld, static_cast<uint32_t>(part_bytes));
        tc::bulk_load(sm, part, static_cast<uint32_t>(part_bytes), bar_ld);
      }
      const bool ok = tc::mbar_wait(bar_ld, ld_phase & 1, WAIT_TIMEOUT_NS);
      const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * HD;
      float* dq_base = a.dqkv + static_cast<int64_t>(b) * S * row_stride + h * HD;
      // DETERMINISM: dQ = (((p0 + p1) + p2) + ...) * scale, as below.
      for (int idx = tid; idx < S * C4 && ok; idx += NB) {
        const int i = idx / C4, c4 = idx % C4;
        const int last = CAUSAL ? min(nkb - 1, i / KB) : nkb - 1;
        float4 v = reinterpret_cast<const float4*>(sp + i * HD)[c4];
        for (int j = 1; j <= last; ++j) {
          const float4 q = reinterpret_cast<const float4*>(sp + (j * S + i) * HD)[c4];
          v = make_float4(v.x + q.x, v.y + q.y, v.z + q.z, v.w + q.w);
        }
        reinterpret_cast<float4*>(dq_base + i * row_stride)[c4] =
            make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
      }
      if (!ok && tid == 0) flag_timeout(a.err, a.sink);
    } else if (s_int[0] == nkb - 1) {
      const float* part = a.dq_part + static_cast<int64_t>(bh) * nkb * S * HD;
      const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * HD;
      float* dq_base = a.dqkv + static_cast<int64_t>(b) * S * row_stride + h * HD;
      // DETERMINISM: dQ = (((p0 + p1) + p2) + ...) * scale over the key blocks holding a key <=
      // the row (causal) or all of them. Eight float4 items per thread at a time, each key
      // block's loads for the eight issued together.
      constexpr int U = 8;
      const int items = S * C4;
      for (int base = tid; base < items; base += U * NB) {
        float4 v[U];
        int last[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int idx = base + u * NB;
          const int i = idx / C4;
          last[u] = idx < items ? (CAUSAL ? min(nkb - 1, i / KB) : nkb - 1) : -1;
          v[u] = last[u] >= 0
                     ? __ldcg(reinterpret_cast<const float4*>(part + static_cast<int64_t>(i) * HD) +
                              (idx % C4))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int j = 1; j < nkb; ++j) {
          float4 p[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int idx = base + u * NB;
            p[u] = j <= last[u] ? __ldcg(reinterpret_cast<const float4*>(
                                             part + (static_cast<int64_t>(j) * S + idx / C4) * HD) +
                                         (idx % C4))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (j <= last[u]) v[u] = make_float4(v[u].x + p[u].x, v[u].y + p[u].y, v[u].z + p[u].z,
                                                 v[u].w + p[u].w);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int idx = base + u * NB;
          if (last[u] >= 0)
            reinterpret_cast<float4*>(dq_base + (idx / C4) * row_stride)[idx % C4] =
                make_float4(v[u].x * a.scale, v[u].y * a.scale, v[u].z * a.scale,
                            v[u].w * a.scale);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (mma_warp) tc::tmem_dealloc(tbase, TMEM_COLS);
}

}  // namespace

cudaError_t setup_bwd_tc_attributes() {
  const void* kernels[] = {reinterpret_cast<const void*>(bwd_tc_kernel<false, 64>),
                           reinterpret_cast<const void*>(bwd_tc_kernel<true, 64>),
                           reinterpret_cast<const void*>(bwd_tc_kernel<false, 32>),
                           reinterpret_cast<const void*>(bwd_tc_kernel<true, 32>)};
  for (const void* k : kernels) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_bwd_tc(const BwdArgs& args, int head_dim, int causal, cudaStream_t stream) {
  BwdArgs a = args;
  a.n_kblocks = (a.S + KB - 1) / KB;
  int dev = 0, sms = 0;  // one block per SM: a wave is the SM count
  if (cudaGetDevice(&dev) == cudaSuccess &&
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
    a.wave_ctas = sms;
  else
    a.wave_ctas = 0;
  const int64_t BH = static_cast<int64_t>(a.B) * a.H;
  const int64_t units = static_cast<int64_t>(a.n_kblocks) * BH;  // key blocks
  int64_t blocks = units;
  // Split tail (non-causal, no-wait dQ path): the R key blocks past the last full wave of P blocks
  // would hold R SMs for a whole block's time while the rest idle; run each as k blocks of
  // consecutive query tiles instead (k = min(tiles, P / R), so they run side by side). The
  // helpers' windows take the part of the dQ-partial region that 128-key blocks leave unused (the
  // workspace sizes it for 64-key blocks), their flags and the tail's ticket counter the turn
  // counters that the no-wait path leaves unused (cleared by the prep kernel). Without room for
  // either, no split.
  a.tail_parts = 0;
  if (a.dq_part != nullptr && !causal && a.wave_ctas > 0) {
    const int64_t P = a.wave_ctas, R = units % P;
    const int64_t n = (a.S + QT - 1) / QT;  // query tiles of every key block
    const int64_t k = R > 0 ? std::min<int64_t>(n, P / R) : 0;
    const int64_t nkb64 = (a.S + BWD_BN - 1) / BWD_BN;  // key blocks the partials are sized for
    const int64_t spare = (nkb64 - a.n_kblocks) * BH * a.S * head_dim;  // floats
    if (k >= 2 && R * n * 2 * KB * head_dim <= spare && BH + R * k + 1 <= BH * a.n_qtiles) {
      a.tail_base = static_cast<int>(units - R);
      a.tail_units = static_cast<int>(R);
      a.tail_parts = static_cast<int>(k);
      a.tail_win = a.dq_part + static_cast<int64_t>(a.n_kblocks) * BH * a.S * head_dim;
      a.tail_flag = a.turn + BH;
      blocks = units - R + R * k;
    }
  }
  const dim3 grid(static_cast<unsigned>(blocks));
  if (head_dim == 32) {
    if (causal) return launch_pdl(bwd_tc_kernel<true, 32>, grid, dim3(NB), SMEM_ALLOC, stream, a);
    return launch_pdl(bwd_tc_kernel<false, 32>, grid, dim3(NB), SMEM_ALLOC, stream, a);
  }
  if (causal) return launch_pdl(bwd_tc_kernel<true, 64>, grid, dim3(NB), SMEM_ALLOC, stream, a);
  return launch_pdl(bwd_tc_kernel<false, 64>, grid, dim3(NB), SMEM_ALLOC, stream, a);
}

}  // namespace cfa
