// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The forward on the tensor cores: O = softmax(Q K^T * scale [+ causal mask]) V and the row
// log-sum-exp L over fp32, head_dim 64 -- the same inputs, outputs and layouts as fwd_ffma.cu and
// the reference's fattn_fwd_f32_d64 (kernels/fused_attn.cu:469-598), computed with tcgen05.mma.
//
// fp32 products from bf16 parts. Every fp32 operand x is split into x0 + x1 + x2, three bf16
// (each part the round-to-nearest bf16 of what the previous ones leave; the two subtractions are
// exact), and A B is formed from the six products A0B0 + (A0B1 + A1B0 + A0B2 + A1B1 + A2B0): the
// dropped terms are below 2^-24 relative. The tensor core accumulates in fp32 by truncation, so
// each product goes to a TMEM accumulator that starts fresh for every window of 64 reduction
// elements (S: all of d; O: one key tile) and takes the five small products of every K-step
// first, the high-order A0B0 steps last: the small sums truncate at their own magnitude (2^-8 of
// the result and below) and only the four A0B0 steps truncate at the result's. Each window's sum
// is added in fp32 registers with round-to-nearest: O = O * alpha + PV per key tile. Modelled
// against fp64 at the canvas shape (baseline/split_precision_model.py) this lands below plain
// sequential-FFMA fp32 on every output of the forward and backward, level with separate
// accumulators for A0B0 and the small products at half the TMEM.
//
// Block: 16 softmax warps and one MMA warp own TC_BM = 128 queries of one (batch, head). Softmax
// thread (warp w < 16, lane l) owns query row 32 (w % 4) + l -- its TMEM lane -- and the 16
// columns (keys of S, dims of O) of group w / 4; warp 16 issues every MMA. The A operands live in
// TMEM -- Q's parts (stored once) for S = Q K^T, P's parts for O = P V -- so an MMA reads only its
// B operand (2 KB) from shared memory and runs at the tensor rate (with both operands in shared
// memory, 6 KB per M128 N64 K16 MMA at 128 B per clock made it 1.5x slower). Per key tile of 64
// the softmax threads read S from TMEM, run the online softmax (row max of the four column groups
// through shared memory), put P's parts into TMEM and split their items of V (transposed: the P V
// product reads V's rows as an MN-major B operand) and K into shared memory; the MMA warp then issues P V(n) and
// S(n + 2). S is issued two tiles ahead (two S buffers in TMEM, two K part buffers) and P V(n - 1)
// is folded into the fp32 O registers one tile late, so the tensor core works while the softmax
// runs. Every thread copies (cp.async) the fp32 chunks it splits itself, a tile ahead of use.
//
// Every mbarrier wait is bounded (WAIT_TIMEOUT_NS); on expiry the block sets the device error flag
// (cfa_fwd_status reads it), waits once more, frees its TMEM and returns without writing.
//
// DETERMINISM: the MMA order is fixed by the code; every register sum has one order: the row
// max over each group's 16 keys in order, then the groups 0..3; p summed over the group's keys in
// order, per tile; l = ((l0 + l1) + l2) + l3; O over key tiles in index order.
#include <cuda_bf16.h>

#include "cfa_common.cuh"
#include "cfa_split.cuh"
#include "cfa_tc.cuh"

namespace cfa {
using tc::kmaj_off;
using tc::split16;
using tc::split8;
using tc::store_parts;
using tc::tmem_ld8;
using tc::tmem_st8;

__device__ int g_fwd_tc_err = 0;

namespace {

constexpr int TC_BM = 128;      // query rows per block = MMA M = TMEM lanes
constexpr int TC_BN = 64;       // keys per tile = MMA N of S = MMA K of P V
constexpr int TC_THREADS = 512;  // the softmax / split threads; one more warp issues the MMAs
constexpr int TC_BLOCK = TC_THREADS + 32;
constexpr int NQ = TC_THREADS / 128;  // threads per query row
constexpr int CW = 64 / NQ;           // columns (keys of S, dims of O) per thread
constexpr int PART_K = TC_BN * 64 * 2;  // bytes of one bf16 part of a [64][64] operand
constexpr int TILE_F32 = TC_BN * 64 * 4;  // bytes of one fp32 [64][64] tile
constexpr int OFF_K = 0;                       // three buffers of K parts, [64 keys][64 d]
constexpr int OFF_V = OFF_K + 9 * PART_K;      // two buffers of V parts, [64 keys][64 d], rows as K's
constexpr int OFF_KST = OFF_V + 6 * PART_K;    // fp32 K tile in flight, [64][64]
constexpr int OFF_VST = OFF_KST + TILE_F32;    // fp32 V tile in flight, [64][64]
constexpr int LDP = 68;                        // prologue staging: rows of 64 floats, 68 apart
constexpr int OFF_ROWS = OFF_VST + TILE_F32;   // prologue: fp32 rows of Q, K(0), K(1)
constexpr int OFF_RED = OFF_ROWS + (TC_BM + 2 * TC_BN) * LDP * 4;  // float [128][NQ]: row max, l
constexpr int OFF_BAR = OFF_RED + TC_BM * NQ * 4;  // mbarriers S0, S1, O, rows; the TMEM base
constexpr int TC_SMEM = OFF_BAR + 40;
constexpr int TC_SMEM_ALLOC = TC_SMEM + 1024;  // room to align the base to 1024 bytes
// TMEM columns (lane = query row). Q's parts, the A operand of S: part i, K-step ks (16 dims) in
// the 8 columns T_Q + 32 i + 8 ks. S of two key tiles (T_S, T_S + 64). O. P's parts, the A operand
// of P V: part i, K-step ks (16 keys) at T_P + 32 i + 8 ks. One block per SM.
constexpr uint32_t T_Q = 0, T_S = 96, T_O = 224, T_P = 288;
constexpr uint32_t TMEM_COLS = 512;

// Staging. Every thread copies (cp.async) exactly the fp32 chunks it later splits, into slots of
// its own, so no barrier separates a copy from its split: a row item (r, kc) -- row r, elements
// 8 kc .. 8 kc + 7 of K or V -- as two 16-byte copies. Slot j of thread t sits at
// (j * TC_THREADS + t) * 16 bytes: a warp's copies and reads of one slot are consecutive.
// Row items: item c takes row 8 (c / 64) + c % 8 and chunk (c / 8) % 8, so a quarter-warp's parts
// land in 8 different bank groups of the core-matrix layout and a warp reads 4 x 32 bytes of each
// of 8 rows.
__device__ __forceinline__ void row_item(int c, int& r, int& kc) {
  r = 8 * (c >> 6) + (c & 7);
  kc = (c >> 3) & 7;
}

// Row item c of the prologue's row-major staging (rows LDP floats apart; rows >= valid read as
// zeros) into K-major parts.
__device__ __forceinline__ void split_staged_row(unsigned char* parts, const float* rows, int c,
                                                 int valid) {
  int r, kc;
  row_item(c, r, kc);
  float x[8];
  if (r < valid) {
    const float4 u = reinterpret_cast<const float4*>(rows + r * LDP + 8 * kc)[0];
    const float4 v = reinterpret_cast<const float4*>(rows + r * LDP + 8 * kc)[1];
    x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = v.x, x[5] = v.y, x[6] = v.z, x[7] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.0f;
  }
  store_parts(parts, PART_K, kmaj_off(r, kc), x);
}

// Copy row item c (slot base `slot`, two 16-byte slots) of a strided operand, rows from r0.
__device__ __forceinline__ void stage_row_item(unsigned char* st, int slot, int c, const float* src,
                                               int64_t stride, int r0, int seq) {
  int r, kc;
  row_item(c, r, kc);
  const bool ok = r0 + r < seq;
  const float* g = src + static_cast<int64_t>(ok ? r0 + r : 0) * stride + 8 * kc;
  cp_async16(st + 16 * ((2 * slot) * TC_THREADS + threadIdx.x), g, ok ? 16 : 0);
  cp_async16(st + 16 * ((2 * slot + 1) * TC_THREADS + threadIdx.x), g + 4, ok ? 16 : 0);
}

__device__ __forceinline__ void split_row_item(unsigned char* parts, int part_bytes,
                                               const unsigned char* st, int slot, int c) {
  int r, kc;
  row_item(c, r, kc);
  const float4 u = *reinterpret_cast<const float4*>(st + 16 * ((2 * slot) * TC_THREADS + threadIdx.x));
  const float4 v =
      *reinterpret_cast<const float4*>(st + 16 * ((2 * slot + 1) * TC_THREADS + threadIdx.x));
  const float x[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
  store_parts(parts, part_bytes, kmaj_off(r, kc), x);
}

// The six (A part, B part) products of K = 64 (four K-steps of 16 bf16) into one accumulator `d`,
// A in TMEM (part i, K-step ks at column a_tmem + 32 i + 8 ks), B in shared memory from b_base:
// the small pairs (0, 1), (1, 0), (0, 2), (1, 1), (2, 0) of every step, then the (0, 0) of every
// step. With A in TMEM an MMA reads only B's 2 KB from shared memory, so it runs at the tensor
// rate. Called by the whole MMA warp (one elected lane issues).
// B is K's parts read K-major (S = Q K^T: K-steps 256 bytes apart) or, B_MN, V's parts -- the same
// row layout -- read MN-major (O = P V, N = d: K-steps of 16 keys 2048 bytes apart).
template <bool B_MN>
__device__ __forceinline__ void issue_split_mma(uint32_t d, uint32_t a_tmem, uint32_t b_base,
                                                uint32_t idesc) {
  constexpr int PA[6] = {0, 0, 1, 0, 1, 2};
  constexpr int PB[6] = {0, 1, 0, 2, 1, 0};
  constexpr int STEP = B_MN ? 2048 : 256;
  const tc::Desc bd = tc::split_desc(B_MN ? tc::desc_kmajor(b_base, 1024, 128)
                                          : tc::desc_kmajor(b_base, 128, 1024));
  const uint32_t id = B_MN ? idesc | (1u << 16) : idesc;
  const uint32_t blo = tc::opaque(bd.lo);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
#pragma unroll
    for (int p = 1; p < 6; ++p)
      tc::mma_bf16_tmem_a_warp(d, a_tmem + 32 * PA[p] + 8 * ks,
                               blo + ((PB[p] * PART_K + STEP * ks) >> 4), bd.hi, id,
                               ks > 0 || p > 1);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
    tc::mma_bf16_tmem_a_warp(d, a_tmem + 8 * ks, blo + ((STEP * ks) >> 4), bd.hi, id, 1);
}

// Named barriers: 2 = the softmax threads plus the MMA warp (TC_BLOCK); 3 + q = the four softmax
// warps of TMEM lane quarter q (w & 3 == q), which hold the same rows and exchange their row maxima.
// Every participant syncs (none only arrives), so no group can run a phase ahead of another even
// when a bounded wait has expired.
__device__ __forceinline__ void bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// CW = 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld1(uint32_t taddr, float (&u)[CW]) {
  static_assert(CW == 16, "one 16-column load per accumulator");
  tc::tmem_ld16(taddr, u);
  tc::tmem_wait_ld();
}

template <bool CAUSAL>
__global__ void __launch_bounds__(TC_BLOCK, 1) fwd_tc_kernel(const FwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* Vp = sm + OFF_V;
  unsigned char* Kst = sm + OFF_KST;
  unsigned char* Vst = sm + OFF_VST;
  float* red = reinterpret_cast<float*>(sm + OFF_RED);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + OFF_BAR);  // [2]
  uint64_t* bar_o = bar_s + 2;
  uint64_t* bar_ld = bar_s + 3;  // the prologue's bulk row copies
  uint32_t* tbase_p = reinterpret_cast<uint32_t*>(bar_s + 4);

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int row = 32 * (w & 3) + lane;  // TMEM lane
  const int cq = w >> 2;                // columns (keys of S, dims of O) CW cq .. CW cq + CW - 1
  const int BH = a.B * a.H;
  int qt, bh;
  if (CAUSAL) {
    qt = a.n_qtiles - 1 - static_cast<int>(blockIdx.x / BH);  // longest tiles first
    bh = static_cast<int>(blockIdx.x % BH);
  } else {
    qt = static_cast<int>(blockIdx.x % a.n_qtiles);
    bh = static_cast<int>(blockIdx.x / a.n_qtiles);
  }
  const int b = bh / a.H, h = bh % a.H;
  const int q0 = qt * TC_BM;
  const int S = a.S;
  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* kp = a.k + b * a.k_sb + h * a.k_sh;
  const float* vp = a.v + b * a.v_sb + h * a.v_sh;
  const int k_end = CAUSAL ? min(S, q0 + TC_BM) : S;
  const int T = (k_end + TC_BN - 1) / TC_BN;  // key tiles, >= 1
  bool err0 = false;

  if (tid == 0) {
    tc::mbar_init(bar_s, 1);
    tc::mbar_init(bar_s + 1, 1);
    tc::mbar_init(bar_o, 1);
    tc::mbar_init(bar_ld, 1);
    tc::fence_mbar_init();
    tc::mbar_arrive_expect_tx(bar_ld, 256u * (min(TC_BM, S - q0) + min(TC_BN, S) +
                                              (T > 1 ? min(TC_BN, S - TC_BN) : 0)));
  }

  griddep_wait();  // q, k, v may come from the previous kernel on the stream
  griddep_launch_dependents();

  // Schedule. Tile n's softmax runs while the tensor core computes P V(n - 1) and S(n + 1): S is
  // issued two tiles ahead (two S buffers in TMEM, three K part buffers), and P V(n - 1) is folded
  // into O one tile late. Per tile n: (a) S(n) -> softmax -> p in registers; (b) P V(n - 1) -> O;
  // (c) p into P's parts; barrier; (d) issue P V(n) and S(n + 2); (e) this thread's items of
  // V(n + 1) and K(n + 3) into their parts (two V buffers, three K buffers: both released) while
  // S(n + 1) completes, then stage V(n + 2), K(n + 4).
  static_assert(TC_BM * 8 == 2 * TC_THREADS && TC_BN * 8 == TC_THREADS, "items per thread");
  const bool mma_warp = w == TC_THREADS / 32;  // warp 16: issues every MMA, nothing else
  // Prologue: the rows of Q, K(0), K(1) travel as one bulk copy each (threads 0-255, one row
  // apiece) into row-major staging (rows past the sequence are not copied and read as zeros),
  // K(2) and V(0) by cp.async; K(0..2), V(0) split into their parts; Q (this thread's row and 16
  // dims: K-step cq of S's A operand) into TMEM; S(0), S(1) issued; V(1), K(3) in flight.
  float* q_rows = reinterpret_cast<float*>(sm + OFF_ROWS);
  float* k_rows = q_rows + TC_BM * LDP;
  const int nq = min(TC_BM, S - q0), nk0 = min(TC_BN, S), nk1 = T > 1 ? min(TC_BN, S - TC_BN) : 0;
  __syncthreads();  // the mbarriers' initialisation
  if (mma_warp) {  // TMEM, by the warp that is idle while the rows travel (it also frees it)
    tc::tmem_alloc(tbase_p, TMEM_COLS);
    tc::tmem_relinquish();
  }
  float qx[CW];
  if (!mma_warp) {
    if (tid < TC_BM) {
      if (tid < nq)
        tc::bulk_load(q_rows + tid * LDP, qp + static_cast<int64_t>(q0 + tid) * a.q_ss, 256, bar_ld);
    } else if (tid < TC_BM + 2 * TC_BN) {
      const int r = tid - TC_BM;  // key row 0 .. 127 of K(0), K(1)
      if (r < (r < TC_BN ? nk0 : TC_BN + nk1))
        tc::bulk_load(k_rows + r * LDP, kp + static_cast<int64_t>(r) * a.k_ss, 256, bar_ld);
    }
    if (T > 2) stage_row_item(Kst, 0, tid, kp, a.k_ss, 2 * TC_BN, S);
    stage_row_item(Vst, 0, tid, vp, a.v_ss, 0, S);
    cp_async_commit();
    err0 = !tc::mbar_wait(bar_ld, 0, WAIT_TIMEOUT_NS);
    cp_async_wait_all();
    split_staged_row(sm + OFF_K, k_rows, tid, nk0);
    if (T > 1) split_staged_row(sm + OFF_K + 3 * PART_K, k_rows + TC_BN * LDP, tid, nk1);
    if (T > 2) split_row_item(sm + OFF_K + 6 * PART_K, PART_K, Kst, 0, tid);
    split_row_item(Vp, PART_K, Vst, 0, tid);
    if (T > 1) stage_row_item(Vst, 0, tid, vp, a.v_ss, TC_BN, S);
    if (T > 3) stage_row_item(Kst, 0, tid, kp, a.k_ss, 3 * TC_BN, S);
    cp_async_commit();
#pragma unroll
    for (int c4 = 0; c4 < CW / 4; ++c4) {
      const float4 u = row < nq ? reinterpret_cast<const float4*>(q_rows + row * LDP + CW * cq)[c4]
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      qx[4 * c4] = u.x;
      qx[4 * c4 + 1] = u.y;
      qx[4 * c4 + 2] = u.z;
      qx[4 * c4 + 3] = u.w;
    }
    tc::fence_async_smem();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tbase_p;
  const uint32_t lane_sel = static_cast<uint32_t>(32 * (w & 3)) << 16;
  const uint32_t t_o = tbase + T_O;
  if (!mma_warp) {
    uint32_t qparts[3][8];
    split16(qx, qparts);
#pragma unroll
    for (int i = 0; i < 3; ++i) tmem_st8(tbase + lane_sel + T_Q + 32 * i + 8 * cq, qparts[i]);
    tc::tmem_wait_st();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  bool err = err0;

  if (mma_warp) {
    // S(0), S(1); then per tile, once its P, V and K(n + 2) parts are in place: P V(n), S(n + 2).
    const uint32_t idesc = tc::idesc_f32acc(1, TC_BM, TC_BN);
    const uint32_t sV = tc::smem_u32(Vp), sK0 = tc::smem_u32(sm + OFF_K);
    // The whole warp runs the issue code (warp-uniform operands); one elected lane issues.
    issue_split_mma<false>(tbase + T_S, tbase + T_Q, sK0, idesc);
    tc::commit_warp(bar_s);
    if (T > 1) {
      issue_split_mma<false>(tbase + T_S + 64, tbase + T_Q, sK0 + 3 * PART_K, idesc);
      tc::commit_warp(bar_s + 1);
    }
    for (int n = 0; n < T; ++n) {
      bar_sync(2, TC_BLOCK);
      tc::fence_after_sync();
      const int j = n & 1;
      issue_split_mma<true>(t_o, tbase + T_P, sV + 3 * PART_K * j, idesc);
      tc::commit_warp(bar_o);
      if (n + 2 < T) {
        issue_split_mma<false>(tbase + T_S + 64 * j, tbase + T_Q, sK0 + 3 * PART_K * ((n + 2) % 3),
                               idesc);
        tc::commit_warp(bar_s + j);
      }
    }
  }

  // The block one wave later (blockIdx + a.wave_ctas) starts by reading its 128 Q rows and the
  // first 128 K rows and 64 V rows of its (batch, head), all at once across the wave: pull them
  // into L2 while this wave computes (one 256-byte row per thread).
  auto prefetch_next_wave = [&]() {
    const int nb = static_cast<int>(blockIdx.x) + a.wave_ctas;
    if (a.wave_ctas <= 0 || nb >= static_cast<int>(gridDim.x) || tid >= 2 * TC_BM + TC_BN) return;
    int nqt, nbh;
    if (CAUSAL) {
      nqt = a.n_qtiles - 1 - nb / BH;
      nbh = nb % BH;
    } else {
      nqt = nb % a.n_qtiles;
      nbh = nb / a.n_qtiles;
    }
    const int nb_b = nbh / a.H, nb_h = nbh % a.H;
    const float* src;
    int r;
    if (tid < TC_BM) {
      r = nqt * TC_BM + tid;
      src = a.q + nb_b * a.q_sb + nb_h * a.q_sh + static_cast<int64_t>(r) * a.q_ss;
    } else if (tid < 2 * TC_BM) {
      r = tid - TC_BM;
      src = a.k + nb_b * a.k_sb + nb_h * a.k_sh + static_cast<int64_t>(r) * a.k_ss;
    } else {
      r = tid - 2 * TC_BM;
      src = a.v + nb_b * a.v_sb + nb_h * a.v_sh + static_cast<int64_t>(r) * a.v_ss;
    }
    if (r < S) asm volatile("cp.async.bulk.prefetch.L2.global [%0], 256;" ::"l"(src) : "memory");
  };

  // Online-softmax state of this thread's columns: acc holds O[row][CW cq + c] (unnormalised).
  float m = -INFINITY, lpart = 0.0f, alpha_prev = 1.0f;
  float acc[CW];
#pragma unroll
  for (int c = 0; c < CW; ++c) acc[c] = 0.0f;
  const int qi = q0 + row;
  float sv[CW];

  // Every softmax thread waits for every commit itself; an expired wait is remembered (the outputs
  // are then invalid) and the block runs on, so all threads keep to the same barriers.
  for (int n = 0; n < T && !mma_warp; ++n) {
    const int k0 = n * TC_BN, j = n & 1;
    // (a) S(n) from TMEM; the online softmax.
    err |= !tc::mbar_wait(bar_s + j, (n >> 1) & 1, WAIT_TIMEOUT_NS);
    tc::fence_after_sync();
    tmem_ld1(tbase + T_S + 64 * j + lane_sel + CW * cq, sv);
    const bool edge = (k0 + TC_BN > S) || (CAUSAL && k0 + TC_BN - 1 > q0);
    float tmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < CW; ++c) {
      float x = sv[c] * a.scale;
      if (edge) {
        const int jj = k0 + CW * cq + c;
        if (!(jj < S && !(CAUSAL && jj > qi))) x = -INFINITY;
      }
      sv[c] = x;
      tmax = fmaxf(tmax, x);
    }
    red[NQ * row + cq] = tmax;
    bar_sync(3 + (w & 3), 32 * NQ);
    tmax = red[NQ * row];
#pragma unroll
    for (int g = 1; g < NQ; ++g) tmax = fmaxf(tmax, red[NQ * row + g]);
    const float m_new = fmaxf(m, tmax);
    const float mu = m_new == -INFINITY ? 0.0f : m_new;  // a fully masked row keeps p = 0
    const float alpha = expf(m - mu);
    float psum = 0.0f;
#pragma unroll
    for (int c = 0; c < CW; ++c) {
      sv[c] = expf(sv[c] - mu);
      psum += sv[c];
    }
    lpart = fmaf(lpart, alpha, psum);
    m = m_new;
    // (b) O += P V(n - 1).
    if (n > 0) {
      err |= !tc::mbar_wait(bar_o, (n - 1) & 1, WAIT_TIMEOUT_NS);
      tc::fence_after_sync();
      float ob[CW];
      tmem_ld1(t_o + lane_sel + CW * cq, ob);
#pragma unroll
      for (int c = 0; c < CW; ++c) acc[c] = fmaf(acc[c], alpha_prev, ob[c]);
    }
    // (c) p into P's parts in TMEM (K-step cq of P V's A operand; P V(n - 1) has read the last
    // ones); hand the tile to the MMA warp.
    {
      uint32_t pparts[3][8];
      split16(sv, pparts);
#pragma unroll
      for (int i = 0; i < 3; ++i) tmem_st8(tbase + lane_sel + T_P + 32 * i + 8 * cq, pparts[i]);
      tc::tmem_wait_st();
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    bar_sync(2, TC_BLOCK);
    tc::fence_after_sync();
    if (n == 0) prefetch_next_wave();
    // (e) While S(n + 1) completes: V(n + 1) into V buffer (n + 1) % 2 (P V(n - 1) has read it) and
    // K(n + 3) into K buffer n % 3 (S(n) has read it) -- both needed at the next hand-off -- then
    // the tiles after them travel.
    cp_async_wait_all();
    if (n + 1 < T) split_row_item(Vp + 3 * PART_K * ((n + 1) & 1), PART_K, Vst, 0, tid);
    if (n + 3 < T) split_row_item(sm + OFF_K + 3 * PART_K * (n % 3), PART_K, Kst, 0, tid);
    tc::fence_async_smem();
    if (n + 2 < T) stage_row_item(Vst, 0, tid, vp, a.v_ss, (n + 2) * TC_BN, S);
    if (n + 4 < T) stage_row_item(Kst, 0, tid, kp, a.k_ss, (n + 4) * TC_BN, S);
    cp_async_commit();
    alpha_prev = alpha;
  }
  if (!mma_warp) {
    // The last tile's P V.
    err |= !tc::mbar_wait(bar_o, (T - 1) & 1, WAIT_TIMEOUT_NS);
    tc::fence_after_sync();
    tmem_ld1(t_o + lane_sel + CW * cq, sv);
#pragma unroll
    for (int c = 0; c < CW; ++c) acc[c] = fmaf(acc[c], alpha_prev, sv[c]);
    cp_async_wait_all();
    red[NQ * row + cq] = lpart;
  }
  if (__syncthreads_or(err)) {
    // A commit did not arrive in time: flag it, give the tensor core one more bounded wait for
    // the last commits, free TMEM, write nothing.
    if (tid == 0) {
      atomicExch(&g_fwd_tc_err, 1);
      flag_timeout(nullptr, a.sink);
    }
    tc::mbar_wait(bar_o, (T - 1) & 1, WAIT_TIMEOUT_NS);
    tc::mbar_wait(bar_s + ((T - 1) & 1), ((T - 1) >> 1) & 1, WAIT_TIMEOUT_NS);
  } else {
    // O = acc / l through shared memory (the K and V part buffers: no MMA is left to read them),
    // rows of LDP floats (a 16-byte rotation per row keeps both passes conflict-free); then every
    // 16 threads store one whole row of O [b, s, h, 64].
    float* o_rows = reinterpret_cast<float*>(sm + OFF_K);
    static_assert(TC_BM * LDP * 4 <= 15 * PART_K, "O rows fit the part buffers");
    if (!mma_warp) {
      float l = red[NQ * row];
#pragma unroll
      for (int g = 1; g < NQ; ++g) l += red[NQ * row + g];
#pragma unroll
      for (int c4 = 0; c4 < CW / 4; ++c4)
        reinterpret_cast<float4*>(o_rows + row * LDP + CW * cq)[c4] =
            make_float4(__fdiv_rn(acc[4 * c4], l), __fdiv_rn(acc[4 * c4 + 1], l),
                        __fdiv_rn(acc[4 * c4 + 2], l), __fdiv_rn(acc[4 * c4 + 3], l));
      if (cq == 0 && qi < S) a.lse[static_cast<int64_t>(bh) * S + qi] = m + logf(l);
    }
    __syncthreads();
    for (int f = tid; f < TC_BM * 16; f += TC_BLOCK) {
      const int r = f >> 4, c4 = f & 15;
      if (q0 + r < S)
        reinterpret_cast<float4*>(a.o + ((static_cast<int64_t>(b) * S + q0 + r) * a.H + h) * 64)[c4] =
            reinterpret_cast<const float4*>(o_rows + r * LDP)[c4];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (mma_warp) tc::tmem_dealloc(tbase, TMEM_COLS);
}

}  // namespace

int fwd_tc_tile_rows() { return TC_BM; }

cudaError_t setup_fwd_tc_attributes() {
  cudaError_t e = cudaFuncSetAttribute(fwd_tc_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_ALLOC);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(fwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              TC_SMEM_ALLOC);
}

cudaError_t launch_fwd_tc(const FwdArgs& args, int causal, cudaStream_t stream) {
  FwdArgs a = args;
  a.n_qtiles = (a.S + TC_BM - 1) / TC_BM;
  int dev = 0, sms = 0;  // one block per SM: a wave is the SM count
  if (cudaGetDevice(&dev) == cudaSuccess &&
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
    a.wave_ctas = sms;
  else
    a.wave_ctas = 0;
  const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(a.n_qtiles) * a.B * a.H));
  if (causal)
    return launch_pdl(fwd_tc_kernel<true>, grid, dim3(TC_BLOCK), TC_SMEM_ALLOC, stream, a);
  return launch_pdl(fwd_tc_kernel<false>, grid, dim3(TC_BLOCK), TC_SMEM_ALLOC, stream, a);
}

cudaError_t fwd_tc_status(int* flag) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_fwd_tc_err, sizeof(int));
  if (e != cudaSuccess) return e;
  *flag = v;
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_fwd_tc_err, &zero, sizeof(int));
  }
  return e;
}

}  // namespace cfa
