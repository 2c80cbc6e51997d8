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
// Block: 256 queries of one (batch, head) as two query tiles of 128 (tile t: rows 128 t ..
// 128 t + 127), 16 softmax warps and one MMA warp. Both tiles read the same K and V parts, so
// every key tile is split into bf16 parts once per 256 queries. The softmax warps work the tiles
// in turn -- softmax of tile 0, then of tile 1, per key tile -- and the tensor core computes one
// tile's P V and next S while the warps run the other tile's softmax (ping-pong): per key tile n,
//   softmax warps:  S0(n) -> P0(n) | split K(n + 2) | S1(n) -> P1(n) | split V(n + 1)
//   MMA warp:       P V0(n), then S0(n + 1) | P V1(n), then S1(n + 1)
// Softmax thread (warp w < 16, lane l) owns query row 32 (w % 4) + l of each tile -- its TMEM lane
// -- and the 16 columns (keys of S, dims of O) of group w / 4; warp 16 issues every MMA.
//
// TMEM (512 columns, lane = query row of the tile). Tile t: Q's parts (the A operand of S = Q K^T,
// written once; part i, K-step ks at T_Q(t) + 32 i + 8 ks), the S / P region (S in its first 64
// columns; after the row's softmax, P's parts over it: part i, K-step ks at T_SP(t) + 32 i +
// 8 ks, the A operand of O = P V) and O (one key tile's P V, folded into registers by the next
// softmax). S(n + 1) overwrites P(n), so it is issued once P V(n) has completed; the other tile's
// work keeps the tensor core busy meanwhile. B operands from shared memory: K's parts K-major,
// V's parts (the same row layout) read MN-major.
//
// Staging. Every thread copies (cp.async) exactly the fp32 chunks of K and V it later splits,
// into slots of its own, so no barrier separates a copy from its split; K(n + 3) and V(n + 2) travel
// while key tile n runs. Three K part buffers, two V part buffers; mbarriers carry every hand-off
// (MMA commits; one arrival per softmax warp for P, K and V parts).
//
// Every mbarrier wait is bounded (WAIT_TIMEOUT_NS); on expiry the block sets the device error flag
// (cfa_fwd_status reads it) and the caller's host-visible flag (cfa_error_sink), waits once more
// for the last commits, frees its TMEM and returns without writing.
//
// DETERMINISM: the MMA order is fixed by the code; every register sum has one order: the row
// max over each group's 16 keys in order, then the groups 0..3; p summed over the group's keys in
// order, per tile; l = ((l0 + l1) + l2) + l3; O over key tiles in index order. A row's arithmetic
// does not depend on the other rows of its block, so results do not depend on the grid.
#include <cuda_bf16.h>

#include <type_traits>

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

constexpr int QT = 128;          // query rows per tile = MMA M = TMEM lanes
constexpr int NTILE = 2;         // query tiles per block
constexpr int BQ = QT * NTILE;   // queries per block
constexpr int KT = 64;           // keys per key tile = MMA N of S = MMA K of P V
constexpr int NSM = 512;         // softmax / split threads; one more warp issues the MMAs
constexpr int NBLK = NSM + 32;
constexpr int NQ = NSM / QT;     // threads per query row
constexpr int CW = 64 / NQ;      // columns (keys of S, dims of O) per thread
constexpr int PART = KT * 64 * 2;   // bytes of one bf16 part of a [64][64] operand
constexpr int PARTS = 3 * PART;     // the three parts of one operand tile
constexpr int STG = NSM * 32;       // one staging set: two 16-byte slots per thread
constexpr int OFF_K = 0;                          // three buffers of K parts, [64 keys][64 d]
constexpr int OFF_V = OFF_K + 3 * PARTS;          // two buffers of V parts, rows as K's
constexpr int OFF_KST = OFF_V + 2 * PARTS;        // fp32 K items in flight
constexpr int OFF_VST = OFF_KST + STG;            // fp32 V items in flight
constexpr int OFF_RED = OFF_VST + STG;            // float [2][128][NQ]: row maxima per tile
constexpr int OFF_LRED = OFF_RED + NTILE * QT * NQ * 4;  // float [2][128][NQ]: row sums
constexpr int OFF_BAR = OFF_LRED + NTILE * QT * NQ * 4;  // mbarriers; the TMEM base
constexpr int NBAR = 11;  // s[2], o[2], p[2], k[2], v[2], q0
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16;
constexpr int SMEM_ALLOC = SMEM + 1024;  // room to align the base to 1024 bytes
constexpr int LDO = 68;  // epilogue: O rows of 64 floats, 68 apart (in the K part buffers)
static_assert(BQ * LDO * 4 <= 3 * PARTS, "the epilogue's O rows fit the K part buffers");
static_assert(STG <= PARTS, "a K part buffer holds one staging set");
static_assert(KT * 8 == NSM, "one K (or V) row item per thread per key tile");
static_assert(SMEM_ALLOC <= 232448, "shared memory per block");

__host__ __device__ constexpr uint32_t T_Q(int t) { return 96u * t; }
__host__ __device__ constexpr uint32_t T_SP(int t) { return 192u + 96u * t; }
__host__ __device__ constexpr uint32_t T_O(int t) { return 384u + 64u * t; }
constexpr uint32_t TMEM_COLS = 512;
static_assert(T_O(1) + 64 == TMEM_COLS, "TMEM budget");

// Row items: item c takes row 8 (c / 64) + c % 8 and chunk (c / 8) % 8 (elements 8 chunk ..
// 8 chunk + 7), so a quarter-warp's parts land in 8 different bank groups of the core-matrix
// layout and a warp reads 4 x 32 bytes of each of 8 rows. Slot j of thread t sits at
// (j * NSM + t) * 16 bytes: a warp's copies and reads of one slot are consecutive.
__device__ __forceinline__ void row_item(int c, int& r, int& kc) {
  r = 8 * (c >> 6) + (c & 7);
  kc = (c >> 3) & 7;
}

// Copy this thread's row item of a strided [seq, HD] operand, rows from r0, as part of a 64-wide
// row (rows past the end and, for HD = 32, chunks past the head dim are zero-filled: source size
// 0, address clamped to row 0).
template <int HD>
__device__ __forceinline__ void stage_item(unsigned char* st, const float* src, int64_t stride,
                                           int r0, int seq) {
  int r, kc;
  row_item(threadIdx.x, r, kc);
  const bool ok = r0 + r < seq && 8 * kc < HD;
  const float* g = src + static_cast<int64_t>(ok ? r0 + r : 0) * stride + 8 * kc;
  cp_async16(st + 16 * threadIdx.x, g, ok ? 16 : 0);
  cp_async16(st + 16 * (NSM + threadIdx.x), g + 4, ok ? 16 : 0);
}

// Q of both query tiles into shared memory for the prologue: 16-byte chunks by consecutive
// threads, so every warp copies whole rows (the rows a thread splits lie 32 rows apart in its
// warp, and read one by one they cost a cache line per thread). Row r (0 .. BQ - 1) at 256 r
// bytes, chunk c at 16 (c ^ (r % 8)): the eight rows a quarter-warp reads in one go fall into
// eight different bank groups. Rows past the end are zero-filled (source size 0).
template <int HD>
__device__ __forceinline__ void stage_q(unsigned char* qs, const float* qp, int64_t stride, int q0,
                                        int seq) {
  constexpr int CPR = HD / 4;  // 16-byte chunks of a row
#pragma unroll
  for (int j = threadIdx.x; j < BQ * CPR; j += NSM) {
    const int r = j / CPR, c = j % CPR;
    const bool ok = q0 + r < seq;
    const float* g = qp + static_cast<int64_t>(ok ? q0 + r : 0) * stride + 4 * c;
    cp_async16(qs + 256 * r + 16 * (c ^ (r & 7)), g, ok ? 16 : 0);
  }
}

// This thread's staged row item into the K-major parts of one operand tile.
__device__ __forceinline__ void split_item(unsigned char* parts, const unsigned char* st) {
  int r, kc;
  row_item(threadIdx.x, r, kc);
  const float4 u = *reinterpret_cast<const float4*>(st + 16 * threadIdx.x);
  const float4 v = *reinterpret_cast<const float4*>(st + 16 * (NSM + threadIdx.x));
  const float x[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
  store_parts(parts, PART, kmaj_off(r, kc), x);
}

// cp.async.wait_group N: every group but the N most recent is complete.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// The six (A part, B part) products of K = 64 (four K-steps of 16 bf16) into one accumulator `d`,
// A in TMEM (part i, K-step ks at column a_tmem + 32 i + 8 ks), B in shared memory from b_base:
// the small pairs (0, 1), (1, 0), (0, 2), (1, 1), (2, 0) of every step, then the (0, 0) of every
// step. With A in TMEM an MMA reads only B's 2 KB from shared memory, so it runs at the tensor
// rate. B is K's parts read K-major (S = Q K^T: K-steps 256 bytes apart) or, B_MN, V's parts --
// the same row layout -- read MN-major (O = P V, N = d: K-steps of 16 keys 2048 bytes apart).
// Called by the whole MMA warp. The 24 MMAs are one asm block: one elect.sync for all of them,
// constant accumulate predicates, and the operand offsets (A: TMEM columns; B: the descriptor's
// start address in 16-byte units, parts PART bytes apart) as immediates -- three instructions an
// MMA, so the issue keeps ahead of the tensor core while the softmax warps share the scheduler.
#define MMA6(AO, BO, P)                                                   \
  "add.u32 at, %1, " #AO ";\n\t"                                          \
  "add.u32 bl, %2, " #BO ";\n\t"                                          \
  "mov.b64 bd, {bl, %3};\n\t"                                             \
  "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [at], bd, %4, " #P ";\n\t"
#define MMA_BLOCK_BEGIN                                                   \
  "{\n\t.reg .pred e, pf, pt;\n\t.reg .b32 at, bl;\n\t.reg .b64 bd;\n\t"  \
  "elect.sync _|e, 0xffffffff;\n\t"                                       \
  "setp.ne.b32 pf, %1, %1;\n\tsetp.eq.b32 pt, %1, %1;\n\t"
static_assert(PART >> 4 == 512, "part stride in descriptor units");

// Head dim 32 (S = Q K^T over 32 dims): the K-steps 0 and 1 of the same window -- the parts of
// K-steps 2 and 3 are zero (the rows are zero-filled past the head dim), and adding exact zeros
// leaves the accumulator unchanged, so these twelve MMAs give the bits of the twenty-four.
__device__ __forceinline__ void issue_split_mma_d32(uint32_t d, uint32_t a_tmem, uint32_t b_base,
                                                    uint32_t idesc) {
  const tc::Desc bd = tc::split_desc(tc::desc_kmajor(b_base, 128, 1024));
  asm volatile(MMA_BLOCK_BEGIN
      MMA6(0, 512, pf)
      MMA6(32, 0, pt)
      MMA6(0, 1024, pt)
      MMA6(32, 512, pt)
      MMA6(64, 0, pt)
      MMA6(8, 528, pt)
      MMA6(40, 16, pt)
      MMA6(8, 1040, pt)
      MMA6(40, 528, pt)
      MMA6(72, 16, pt)
      MMA6(0, 0, pt)
      MMA6(8, 16, pt)
      "}\n" ::"r"(d), "r"(a_tmem), "r"(bd.lo), "r"(bd.hi), "r"(idesc)
      : "memory");
}

template <bool B_MN>
__device__ __forceinline__ void issue_split_mma(uint32_t d, uint32_t a_tmem, uint32_t b_base,
                                                uint32_t idesc) {
  const tc::Desc bd = tc::split_desc(B_MN ? tc::desc_kmajor(b_base, 1024, 128)
                                          : tc::desc_kmajor(b_base, 128, 1024));
  const uint32_t id = B_MN ? idesc | (1u << 16) : idesc;
  if constexpr (!B_MN) {
    asm volatile(MMA_BLOCK_BEGIN
        MMA6(0, 512, pf)
        MMA6(32, 0, pt)
        MMA6(0, 1024, pt)
        MMA6(32, 512, pt)
        MMA6(64, 0, pt)
        MMA6(8, 528, pt)
        MMA6(40, 16, pt)
        MMA6(8, 1040, pt)
        MMA6(40, 528, pt)
        MMA6(72, 16, pt)
        MMA6(16, 544, pt)
        MMA6(48, 32, pt)
        MMA6(16, 1056, pt)
        MMA6(48, 544, pt)
        MMA6(80, 32, pt)
        MMA6(24, 560, pt)
        MMA6(56, 48, pt)
        MMA6(24, 1072, pt)
        MMA6(56, 560, pt)
        MMA6(88, 48, pt)
        MMA6(0, 0, pt)
        MMA6(8, 16, pt)
        MMA6(16, 32, pt)
        MMA6(24, 48, pt)
        "}\n" ::"r"(d), "r"(a_tmem), "r"(bd.lo), "r"(bd.hi), "r"(id)
        : "memory");
  } else {
    asm volatile(MMA_BLOCK_BEGIN
        MMA6(0, 512, pf)
        MMA6(32, 0, pt)
        MMA6(0, 1024, pt)
        MMA6(32, 512, pt)
        MMA6(64, 0, pt)
        MMA6(8, 640, pt)
        MMA6(40, 128, pt)
        MMA6(8, 1152, pt)
        MMA6(40, 640, pt)
        MMA6(72, 128, pt)
        MMA6(16, 768, pt)
        MMA6(48, 256, pt)
        MMA6(16, 1280, pt)
        MMA6(48, 768, pt)
        MMA6(80, 256, pt)
        MMA6(24, 896, pt)
        MMA6(56, 384, pt)
        MMA6(24, 1408, pt)
        MMA6(56, 896, pt)
        MMA6(88, 384, pt)
        MMA6(0, 0, pt)
        MMA6(8, 128, pt)
        MMA6(16, 256, pt)
        MMA6(24, 384, pt)
        "}\n" ::"r"(d), "r"(a_tmem), "r"(bd.lo), "r"(bd.hi), "r"(id)
        : "memory");
  }
}
#undef MMA6
#undef MMA_BLOCK_BEGIN

// Named barriers 3 + q: the four softmax warps of TMEM lane quarter q (w % 4 == q), which hold
// the same rows and exchange their row maxima. Every participant syncs, so no warp can run a
// phase ahead of another even when a bounded wait has expired.
__device__ __forceinline__ void bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// The limit of a thread's next mbarrier wait: WAIT_TIMEOUT_NS, or 1 ms once one of its waits has
// expired (the results are invalid by then; the block only has to reach its end quickly, every
// thread still keeping to the same arrivals and barriers).
__device__ __forceinline__ uint64_t wait_ns(bool expired) {
  return expired ? 1000000ull : WAIT_TIMEOUT_NS;
}

// Packed fp32 pairs (tc::pack2 / unpack2): products, sums and the O fold one instruction a pair.
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// (x, y) = (x, y) * a + b, one rounding per lane.
__device__ __forceinline__ void fma2x(float& x, float& y, uint64_t a, uint64_t b) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(tc::pack2(x, y)), "l"(a), "l"(b));
  tc::unpack2(d, x, y);
}
constexpr float LOG2E = 1.4426950408889634f;  // log2(e), rounded to fp32

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void tmem_ld1(uint32_t taddr, float (&u)[CW]) {
  static_assert(CW == 16, "one 16-column load per accumulator");
  tc::tmem_ld16(taddr, u);
  tc::tmem_wait_ld();
}

// The online-softmax state of one thread for one query tile: its 16 columns of O (unnormalised),
// the row maximum m of the scaled scores, its share of the row sum, and the last tile's rescale
// factor.
struct RowState {
  float acc[CW];
  float m, lpart, alpha_prev;
};

template <bool CAUSAL, int HD>
__global__ void __launch_bounds__(NBLK, 1) fwd_tc_kernel(const FwdArgs a) {
  static_assert(HD == 64 || HD == 32, "head dims of the tensor-core forward");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* Kp = sm + OFF_K;
  unsigned char* Vp = sm + OFF_V;
  unsigned char* Kst = sm + OFF_KST;
  unsigned char* Vst = sm + OFF_VST;
  float* red = reinterpret_cast<float*>(sm + OFF_RED);
  float* lred = reinterpret_cast<float*>(sm + OFF_LRED);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + OFF_BAR);  // [2]: S(t) committed
  uint64_t* bar_o = bar_s + 2;  // [2]: P V(t) committed
  uint64_t* bar_p = bar_s + 4;  // [2]: P(t)'s parts in TMEM (one arrival per softmax warp)
  uint64_t* bar_k = bar_s + 6;  // [2]: K(j)'s parts in place, j >= 2, by j % 2 (same)
  uint64_t* bar_v = bar_s + 8;  // [2]: V(j)'s parts in place, j >= 1, by j % 2 (same)
  uint64_t* bar_q0 = bar_s + 10;  // Q's parts in TMEM and K(0)'s in place (same)
  uint32_t* tbase_p = reinterpret_cast<uint32_t*>(bar_s + NBAR);

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const bool mma_warp = w == NSM / 32;  // warp 16: issues every MMA, nothing else
  const int row = 32 * (w & 3) + lane;  // TMEM lane: query row of each tile
  const int cq = w >> 2;                // columns CW cq .. CW cq + CW - 1
  const int BH = a.B * a.H;
  int qb, bh;
  if (CAUSAL) {
    qb = a.n_qtiles - 1 - static_cast<int>(blockIdx.x / BH);  // longest blocks first
    bh = static_cast<int>(blockIdx.x % BH);
  } else {
    qb = static_cast<int>(blockIdx.x % a.n_qtiles);
    bh = static_cast<int>(blockIdx.x / a.n_qtiles);
  }
  const int b = bh / a.H, h = bh % a.H;
  const int q0 = qb * BQ;
  const int S = a.S;
  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* kp = a.k + b * a.k_sb + h * a.k_sh;
  const float* vp = a.v + b * a.v_sb + h * a.v_sh;
  // Key tiles of each query tile (0: the tile lies past the sequence), and of the block.
  int Tt[NTILE];
#pragma unroll
  for (int t = 0; t < NTILE; ++t) {
    const int r0 = q0 + QT * t;
    const int k_end = CAUSAL ? min(S, r0 + QT) : S;
    Tt[t] = r0 < S ? (k_end + KT - 1) / KT : 0;
  }
  const int T0 = Tt[0], T1 = Tt[1];
  const int T = max(T0, T1);  // >= 1

  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < NBAR; ++i) tc::mbar_init(bar_s + i, i < 4 ? 1 : NSM / 32);  // q0: 16
    tc::fence_mbar_init();
  }
  griddep_wait();  // q, k, v may come from the previous kernel on the stream
  griddep_launch_dependents();
  __syncthreads();  // the mbarriers' initialisation
  if (mma_warp) {  // TMEM, by the warp that issues the MMAs (it also frees it)
    tc::tmem_alloc(tbase_p, TMEM_COLS);
    tc::tmem_relinquish();
  }

  // Prologue: Q of both tiles staged over K part buffers 1 and 2 and the first 16 KB of V part
  // buffer 0 (stage_q), K(0), K(1), V(0) as row items (K(1) in V part buffer 1, free until the
  // first loop step). K(0) into its parts (buffer 0, clear of the staged Q) and Q (this thread's row and 16
  // dims: K-step cq of S's A operand) into TMEM release the first S at once (bar_q0); K(1), V(0)
  // go into their parts -- over the staged Q, once every thread has read its rows -- while the
  // tensor core runs it: every softmax thread has split them before its first P arrival, which
  // the MMA warp awaits before the first P V and S(1). K(2), V(1) are left in flight.
  unsigned char* qst = Kp + PARTS;
  static_assert(PARTS + BQ * 256 <= OFF_V - OFF_K + PARTS, "the staged Q ends inside V part buffer 0");
  if (!mma_warp) {
    stage_q<HD>(qst, qp, a.q_ss, q0, S);
    stage_item<HD>(Kst, kp, a.k_ss, 0, S);
    if (T > 1) stage_item<HD>(Vp + PARTS, kp, a.k_ss, KT, S);
    stage_item<HD>(Vst, vp, a.v_ss, 0, S);
    cp_async_commit();
  }
  tc::fence_before_sync();
  __syncthreads();  // the TMEM base
  tc::fence_after_sync();
  const uint32_t tbase = *tbase_p;
  const uint32_t lane_sel = static_cast<uint32_t>(32 * (w & 3)) << 16;
  if (!mma_warp) {
    cp_async_wait_all();
    split_item(Kp, Kst);  // K(0)
    tc::fence_async_smem();
    bar_sync(1, NSM);  // every thread's share of Q in place
#pragma unroll
    for (int t = 0; t < NTILE; ++t) {
      const int r = QT * t + row;
      float qx[CW];
#pragma unroll
      for (int c4 = 0; c4 < CW / 4; ++c4) {
        const float4 u = CW * cq < HD ? *reinterpret_cast<const float4*>(
                                            qst + 256 * r + 16 * ((CW / 4 * cq + c4) ^ (r & 7)))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        qx[4 * c4] = u.x;
        qx[4 * c4 + 1] = u.y;
        qx[4 * c4 + 2] = u.z;
        qx[4 * c4 + 3] = u.w;
      }
      uint32_t qparts[3][8];
      split16(qx, qparts);
#pragma unroll
      for (int i = 0; i < 3; ++i) tmem_st8(tbase + lane_sel + T_Q(t) + 32 * i + 8 * cq, qparts[i]);
    }
    tc::tmem_wait_st();
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(bar_q0);  // the first S may start
    bar_sync(1, NSM);  // every thread has read its Q rows: the buffers under the staged Q are free
    if (T > 1) split_item(Kp + PARTS, Vp + PARTS);  // K(1)
    split_item(Vp, Vst);                            // V(0)
    tc::fence_async_smem();
    // Every thread's K(1) staging slots read before any V(1) part lands on them (split_v(0)).
    bar_sync(1, NSM);
    // In flight during key tile 0: K(2), then V(1) (two cp.async groups, in that order), issued
    // while the tensor core computes the first S (each thread reuses staging slots only it read).
    if (T > 2) stage_item<HD>(Kst, kp, a.k_ss, 2 * KT, S);
    cp_async_commit();
    if (T > 1) stage_item<HD>(Vst, vp, a.v_ss, KT, S);
    cp_async_commit();
  }
  bool err = false;

  if (mma_warp) {
    // Per key tile n and tile t: once P(t, n) is in TMEM (and V(n) in place), P V(t, n); once that
    // has completed -- S(t, n + 1) overwrites P(t, n) -- and K(n + 1) is in place, S(t, n + 1).
    // The whole warp runs the issue code (warp-uniform operands); one elected lane issues.
    const uint32_t idesc = tc::idesc_f32acc(1, QT, KT);     // S: N = 64 keys
    const uint32_t idesc_pv = tc::idesc_f32acc(1, QT, HD);  // P V: N = the head dim
    const uint32_t sK = tc::smem_u32(Kp), sV = tc::smem_u32(Vp);
    err |= !tc::mbar_wait(bar_q0, 0, wait_ns(err));  // Q in TMEM, K(0)'s parts in place
    tc::fence_after_sync();
#pragma unroll
    for (int t = 0; t < NTILE; ++t)
      if (Tt[t] > 0) {
        if constexpr (HD == 32) issue_split_mma_d32(tbase + T_SP(t), tbase + T_Q(t), sK, idesc);
        else issue_split_mma<false>(tbase + T_SP(t), tbase + T_Q(t), sK, idesc);
        tc::commit_warp(bar_s + t);
      }
    for (int n = 0; n < T; ++n) {
      bool v_ready = n == 0, k_ready = n + 1 < 2;
#pragma unroll
      for (int t = 0; t < NTILE; ++t) {
        if (n >= Tt[t]) continue;
        err |= !tc::mbar_wait(bar_p + t, n & 1, wait_ns(err));
        if (!v_ready) {  // V(n), n >= 1: completion (n - 1) / 2 of bar_v[n % 2]
          err |= !tc::mbar_wait(bar_v + (n & 1), ((n - 1) >> 1) & 1, wait_ns(err));
          v_ready = true;
        }
        tc::fence_after_sync();
        issue_split_mma<true>(tbase + T_O(t), tbase + T_SP(t), sV + PARTS * (n & 1), idesc_pv);
        tc::commit_warp(bar_o + t);
        if (n + 1 < Tt[t]) {
          err |= !tc::mbar_wait(bar_o + t, n & 1, wait_ns(err));
          if (!k_ready) {  // K(n + 1), n + 1 >= 2: completion (n - 1) / 2 of bar_k[(n + 1) % 2]
            err |= !tc::mbar_wait(bar_k + ((n + 1) & 1), ((n - 1) >> 1) & 1, wait_ns(err));
            k_ready = true;
          }
          tc::fence_after_sync();
          if constexpr (HD == 32)
            issue_split_mma_d32(tbase + T_SP(t), tbase + T_Q(t), sK + PARTS * ((n + 1) % 3), idesc);
          else
            issue_split_mma<false>(tbase + T_SP(t), tbase + T_Q(t), sK + PARTS * ((n + 1) % 3),
                                   idesc);
          tc::commit_warp(bar_s + t);
        }
      }
    }
  }

  // The block one wave later (blockIdx + a.wave_ctas) starts by reading its 256 Q rows and the
  // first 128 K rows and 64 V rows of its (batch, head): pull them into L2 while this wave
  // computes (one 256-byte row per thread).
  auto prefetch_next_wave = [&]() {
    const int nb = static_cast<int>(blockIdx.x) + a.wave_ctas;
    if (a.wave_ctas <= 0 || nb >= static_cast<int>(gridDim.x) || tid >= BQ + 2 * KT + KT) return;
    int nqb, nbh;
    if (CAUSAL) {
      nqb = a.n_qtiles - 1 - nb / BH;
      nbh = nb % BH;
    } else {
      nqb = nb % a.n_qtiles;
      nbh = nb / a.n_qtiles;
    }
    const int nb_b = nbh / a.H, nb_h = nbh % a.H;
    const float* src;
    int r;
    if (tid < BQ) {
      r = nqb * BQ + tid;
      src = a.q + nb_b * a.q_sb + nb_h * a.q_sh + static_cast<int64_t>(r) * a.q_ss;
    } else if (tid < BQ + 2 * KT) {
      r = tid - BQ;
      src = a.k + nb_b * a.k_sb + nb_h * a.k_sh + static_cast<int64_t>(r) * a.k_ss;
    } else {
      r = tid - BQ - 2 * KT;
      src = a.v + nb_b * a.v_sb + nb_h * a.v_sh + static_cast<int64_t>(r) * a.v_ss;
    }
    if (r < S) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "n"(4 * HD) : "memory");
  };

  const uint64_t sc2 = tc::pack2(a.scale, a.scale);
  const uint64_t l2e2 = tc::pack2(LOG2E, LOG2E);
  RowState st[NTILE];
#pragma unroll
  for (int t = 0; t < NTILE; ++t) {
    st[t].m = -INFINITY;
    st[t].lpart = 0.0f;
    st[t].alpha_prev = 1.0f;
#pragma unroll
    for (int c = 0; c < CW; ++c) st[t].acc[c] = 0.0f;
  }

  // Key tile n of query tile t: fold P V(t, n - 1) into O (it uses the previous tile's rescale
  // factor only, so it comes first and its TMEM values never share registers with S's), then the
  // online softmax of S(t, n) into P(t, n)'s parts; for n == Tt[t], only that last fold. Every
  // softmax thread waits for every commit itself; an expired wait is remembered (the outputs are
  // then invalid) and the block runs on, so all threads keep to the same barriers.
  auto softmax_step = [&](auto tile, int n) {
    constexpr int t = decltype(tile)::value;
    RowState& rs = st[t];
    const int Tn = Tt[t];
    if (n > Tn) return;
    if (n > 0) {  // O = O * alpha(n - 1) + P V(t, n - 1)
      err |= !tc::mbar_wait(bar_o + t, (n - 1) & 1, wait_ns(err));
      tc::fence_after_sync();
      if (CW * cq < HD) {  // O has HD columns
        float ob[CW];
        tmem_ld1(tbase + lane_sel + T_O(t) + CW * cq, ob);
        const uint64_t al2 = tc::pack2(rs.alpha_prev, rs.alpha_prev);
#pragma unroll
        for (int c = 0; c < CW; c += 2)
          fma2x(rs.acc[c], rs.acc[c + 1], al2, tc::pack2(ob[c], ob[c + 1]));
      }
    }
    if (n == Tn) return;
    const int k0 = n * KT;
    const int qi = q0 + QT * t + row;
    float sv[CW];
    err |= !tc::mbar_wait(bar_s + t, n & 1, wait_ns(err));
    tc::fence_after_sync();
    tmem_ld1(tbase + lane_sel + T_SP(t) + CW * cq, sv);
    // Scaled scores y = s * scale, masked to -inf past the end / diagonal.
#pragma unroll
    for (int c = 0; c < CW; c += 2) {
      const uint64_t y = mul2(tc::pack2(sv[c], sv[c + 1]), sc2);
      tc::unpack2(y, sv[c], sv[c + 1]);
    }
    const bool edge = (k0 + KT > S) || (CAUSAL && k0 + KT - 1 > q0 + QT * t);
    if (edge) {
#pragma unroll
      for (int c = 0; c < CW; ++c) {
        const int jj = k0 + CW * cq + c;
        if (!(jj < S && !(CAUSAL && jj > qi))) sv[c] = -INFINITY;
      }
    }
    float tmax = max3f(sv[0], sv[1], sv[2]);
#pragma unroll
    for (int c = 3; c < CW - 1; c += 2) tmax = max3f(tmax, sv[c], sv[c + 1]);
    tmax = fmaxf(tmax, sv[CW - 1]);
    float* rr = red + (t * QT + row) * NQ;
    rr[cq] = tmax;
    tc::fence_before_sync();  // every S read of the row done before any thread stores P over it
    bar_sync(3 + (w & 3), 32 * NQ);
    tc::fence_after_sync();
    tmax = max3f(max3f(rs.m, rr[0], rr[1]), rr[2], rr[3]);
    const float mu = tmax == -INFINITY ? 0.0f : tmax;  // a fully masked row keeps p = 0
    // e^(y - mu) = 2^((y - mu) log2 e): y - mu is exact where p matters (Sterbenz), one rounding
    // of the product, then the SFU's 2^x (ex2.approx, max relative error about 2^-22).
    const float alpha = ex2((rs.m - mu) * LOG2E);
    const uint64_t mu2 = tc::pack2(mu, mu);
    uint64_t ps2 = 0;  // (+0, +0)
    // p into P's parts in TMEM (K-step cq of P V's A operand), in two halves of 8 keys (columns
    // 4 h .. 4 h + 3 of the K-step): each half's stores travel while the next half is formed.
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
      for (int c = 8 * hh; c < 8 * hh + 8; c += 2) {
        float lo, hi;
        tc::unpack2(mul2(tc::sub2(tc::pack2(sv[c], sv[c + 1]), mu2), l2e2), lo, hi);
        sv[c] = ex2(lo);
        sv[c + 1] = ex2(hi);
        ps2 = add2(ps2, tc::pack2(sv[c], sv[c + 1]));
      }
      const float xh[8] = {sv[8 * hh], sv[8 * hh + 1], sv[8 * hh + 2], sv[8 * hh + 3],
                           sv[8 * hh + 4], sv[8 * hh + 5], sv[8 * hh + 6], sv[8 * hh + 7]};
      uint4 h0, h1, h2;
      split8(xh, h0, h1, h2);
      const uint32_t pc = tbase + lane_sel + T_SP(t) + 8 * cq + 4 * hh;
      tc::tmem_st4(pc, h0);
      tc::tmem_st4(pc + 32, h1);
      tc::tmem_st4(pc + 64, h2);
    }
    float ps_lo, ps_hi;
    tc::unpack2(ps2, ps_lo, ps_hi);
    rs.lpart = fmaf(rs.lpart, alpha, ps_lo + ps_hi);
    rs.m = tmax;
    rs.alpha_prev = alpha;
    // Hand the tile to the MMA warp.
    tc::tmem_wait_st();
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(bar_p + t);
  };

  // K(n + 2) into K buffer (n + 2) % 3 (it held K(n - 1): S(0, n - 1), S(1, n - 1) have completed),
  // then K(n + 3) travels. It runs after a softmax step that waited for S(t, n) of an active tile:
  // the MMA warp issued that S after waiting for K(n), so bar_k[n % 2] never completes K(n + 2)
  // before the MMA warp has seen K(n) complete.
  auto split_k = [&](int n) {
    cp_async_wait_group<1>();  // K(n + 2)'s group (V(n + 1)'s, committed after it, may remain)
    if (n + 2 < T) {
      split_item(Kp + PARTS * ((n + 2) % 3), Kst);
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_k + (n & 1));
    }
    if (n + 3 < T) stage_item<HD>(Kst, kp, a.k_ss, (n + 3) * KT, S);
    cp_async_commit();
  };
  // V(n + 1) into V buffer (n + 1) % 2 (it held V(n - 1): both P V(t, n - 1) have completed --
  // each thread has waited for them in this step's folds), then V(n + 2) travels.
  auto split_v = [&](int n) {
    cp_async_wait_group<1>();
    if (n + 1 < T) {
      split_item(Vp + PARTS * ((n + 1) & 1), Vst);
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_v + ((n + 1) & 1));
    }
    if (n + 2 < T) stage_item<HD>(Vst, vp, a.v_ss, (n + 2) * KT, S);
    cp_async_commit();
  };

  if (!mma_warp) {
    for (int n = 0; n <= T; ++n) {
      softmax_step(std::integral_constant<int, 0>{}, n);
      if (n == 0) prefetch_next_wave();
      if (n < T0) split_k(n);  // tile 0 waited for S(0, n)
      softmax_step(std::integral_constant<int, 1>{}, n);
      if (n >= T0) split_k(n);  // tile 0 done (causal tail): tile 1 waited for S(1, n)
      split_v(n);
    }
    cp_async_wait_all();
#pragma unroll
    for (int t = 0; t < NTILE; ++t) lred[(t * QT + row) * NQ + cq] = st[t].lpart;
  }
  if (__syncthreads_or(err)) {
    // A commit did not arrive in time: flag it, give the tensor core one more bounded wait for
    // the last commits, free TMEM, write nothing.
    if (tid == 0) {
      atomicExch(&g_fwd_tc_err, 1);
      flag_timeout(nullptr, a.sink);
    }
#pragma unroll
    for (int t = 0; t < NTILE; ++t)
      if (Tt[t] > 0) tc::mbar_wait(bar_o + t, (Tt[t] - 1) & 1, WAIT_TIMEOUT_NS);
  } else {
    // O = acc * (1 / l) through shared memory (the K part buffers: every MMA has completed), rows of
    // LDO floats (a 16-byte rotation per row keeps both passes conflict-free); then every 16
    // threads store one whole row of O [b, s, h, 64].
    float* o_rows = reinterpret_cast<float*>(sm + OFF_K);
    if (!mma_warp) {
#pragma unroll
      for (int t = 0; t < NTILE; ++t) {
        const float* lr = lred + (t * QT + row) * NQ;
        float l = lr[0];
#pragma unroll
        for (int g = 1; g < NQ; ++g) l += lr[g];
        float* orow = o_rows + (t * QT + row) * LDO + CW * cq;
        // O = acc * RN(1 / l): one IEEE reciprocal a row, then products (a rounding more than a
        // division per element, 4 µs less per canvas forward; O stays below the FFMA pair's error).
        const float rl = __frcp_rn(l);
#pragma unroll
        for (int c4 = 0; c4 < CW / 4; ++c4)
          reinterpret_cast<float4*>(orow)[c4] =
              make_float4(st[t].acc[4 * c4] * rl, st[t].acc[4 * c4 + 1] * rl,
                          st[t].acc[4 * c4 + 2] * rl, st[t].acc[4 * c4 + 3] * rl);
        const int qi = q0 + QT * t + row;
        if (cq == 0 && qi < S) a.lse[static_cast<int64_t>(bh) * S + qi] = st[t].m + logf(l);
      }
    }
    __syncthreads();
    constexpr int C4 = HD / 4;  // float4 columns of an O row [b, s, h, HD]
    for (int f = tid; f < BQ * C4; f += NBLK) {
      const int r = f / C4, c4 = f % C4;
      if (q0 + r < S)
        reinterpret_cast<float4*>(a.o + ((static_cast<int64_t>(b) * S + q0 + r) * a.H + h) * HD)[c4] =
            reinterpret_cast<const float4*>(o_rows + r * LDO)[c4];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (mma_warp) tc::tmem_dealloc(tbase, TMEM_COLS);
}

}  // namespace

cudaError_t setup_fwd_tc_attributes() {
  const void* kernels[] = {reinterpret_cast<const void*>(fwd_tc_kernel<false, 64>),
                           reinterpret_cast<const void*>(fwd_tc_kernel<true, 64>),
                           reinterpret_cast<const void*>(fwd_tc_kernel<false, 32>),
                           reinterpret_cast<const void*>(fwd_tc_kernel<true, 32>)};
  for (const void* k : kernels) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_fwd_tc(const FwdArgs& args, int head_dim, int causal, cudaStream_t stream) {
  FwdArgs a = args;
  a.n_qtiles = (a.S + BQ - 1) / BQ;  // blocks of 256 queries per (batch, head)
  int dev = 0, sms = 0;  // one block per SM: a wave is the SM count
  if (cudaGetDevice(&dev) == cudaSuccess &&
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
    a.wave_ctas = sms;
  else
    a.wave_ctas = 0;
  const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(a.n_qtiles) * a.B * a.H));
  if (head_dim == 32) {
    if (causal) return launch_pdl(fwd_tc_kernel<true, 32>, grid, dim3(NBLK), SMEM_ALLOC, stream, a);
    return launch_pdl(fwd_tc_kernel<false, 32>, grid, dim3(NBLK), SMEM_ALLOC, stream, a);
  }
  if (causal) return launch_pdl(fwd_tc_kernel<true, 64>, grid, dim3(NBLK), SMEM_ALLOC, stream, a);
  return launch_pdl(fwd_tc_kernel<false, 64>, grid, dim3(NBLK), SMEM_ALLOC, stream, a);
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
