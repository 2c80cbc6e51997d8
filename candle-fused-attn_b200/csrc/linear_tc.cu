// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The projection next to the attention on the tensor cores: C = A B over fp32, the contraction of
// candle's `broadcast_matmul` in the reference's training step (examples/tutorial.rs:103-118:
// qkv = x W_qkv feeds fused_attention_qkv, and the step's gradient of W_qkv is x^T dqkv). Any
// orientation: A(m, k) and B(k, n) are read through (row, column) strides (any values), so x W,
// dY W^T and x^T dY all run on this kernel without a transposed copy.
//
// fp32 products from bf16 parts, as in the attention kernels: every fp32 operand x is split into
// x0 + x1 + x2, three bf16 (each part the round-to-nearest bf16 of what the previous ones leave;
// both subtractions exact), and A B is formed from the six products A0B0 + (A0B1 + A1B0 + A0B2 +
// A1B1 + A2B0); the dropped terms are below 2^-24 relative. The tensor core accumulates by
// truncation, so the products go to two TMEM accumulators that start fresh every window of 64
// reduction elements: `hi` takes the four A0B0 steps, `lo` the twenty small products (2^-8 of the
// result and below, so they truncate at their own magnitude). Each window's hi + lo is added into
// fp32 registers with round-to-nearest, windows in K order.
//
// Two kernels. The split kernel writes each operand once, as bf16 parts, into the workspace in
// the exact layout the MMA reads: blocks of 128 rows (M or N) x 16 K, three 4 KB parts each,
// K-major no-swizzle core matrices -- whatever the operand's strides (transposed views and x^T
// need no copy). The product kernel then does no CUDA-core work on the operands (one block per
// SM, persistent; output tiles of 128 x 128):
//  - producer warp: one lane issues two bulk copies per ring slot (two K-steps of A's blocks and
//    of B's, 48 KB) into a ring of NSLOT slots, eight K-steps ahead of the tensor core;
//  - MMA warp: twelve MMAs per slot (M = N = 128, A and B from shared memory) from two asm blocks
//    with the wait for the next slot between them, a commit per slot, and one per window into the
//    window's accumulator pair (two pairs: 512 TMEM columns), so the tensor core runs one window
//    while the fold warps read the last;
//  - fold warps: thread (lane quarter q, column half h) adds each window's hi + lo of row 32 q +
//    lane, columns 64 h .. + 63, into its 64 running sums and, after an output tile's last
//    window, writes them through a per-warp staging block as whole 128-byte rows.
// Work items are (output tile, K chunk): when the output has fewer tiles than the GPU has SMs, K is
// cut into chunks whose partial tiles a second kernel sums in chunk order. The chunk count is a
// function of (M, N, K) alone, and every item's arithmetic is independent of where it runs, so the
// result is bit-identical across reruns, grid sizes and GPUs.
//
// Every mbarrier wait is bounded (WAIT_TIMEOUT_NS, then 1 ms once one has expired); on expiry the
// block sets the device error flag (cfa_matmul_status reads it) and the host-visible flag
// (cfa_error_sink), keeps to every arrival, frees its TMEM and writes nothing more.
#include <cuda_bf16.h>

#include <algorithm>

#include "cfa_common.cuh"
#include "cfa_split.cuh"
#include "cfa_tc.cuh"

namespace cfa {

__device__ int g_linear_err = 0;

namespace {

constexpr int TM = 128;          // output rows per tile = MMA M = TMEM lanes
constexpr int TN = 128;          // output columns per tile = MMA N
constexpr int KS = 16;           // K per MMA step
constexpr int WIN_STEPS = 4;     // K-steps per accumulation window (64 reduction elements)
constexpr int PART = TM * KS * 2;        // one bf16 part of a 128 x 16 operand block
constexpr int BLOCK = 3 * PART;          // the three parts of one operand block
constexpr int SLOT_STEPS = 2;            // K-steps per ring slot
constexpr int SLOT = 2 * SLOT_STEPS * BLOCK;  // a ring slot: A's two blocks, then B's
constexpr int NSLOT = 4;                 // ring slots (two windows)
constexpr int NFOLD = 256;               // fold threads (warps 0-7)
constexpr int PRODUCER_WARP = NFOLD / 32;
constexpr int MMA_WARP = PRODUCER_WARP + 1;
constexpr int NTHR = NFOLD + 64;
constexpr int FC = TN * TM / NFOLD;      // output columns per fold thread
constexpr int OFF_OUT = NSLOT * SLOT;   // per fold warp: a 32 x 32 fp32 staging block (4 KB)
constexpr int OUT_WARP = 32 * 32 * 4;
constexpr int OFF_BAR = OFF_OUT + (NFOLD / 32) * OUT_WARP;
constexpr int NBAR = 2 * NSLOT + 4;      // full[NSLOT], empty[NSLOT], accf[2], acce[2]
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16;
constexpr int SMEM_ALLOC = SMEM + 128;   // room to align the base to 128 bytes
constexpr uint32_t TMEM_COLS = 512;      // accumulator pair b: hi at 256 b, lo at 256 b + 128
constexpr int SPLIT_THREADS = 256;       // one 8-element item of a block per thread
static_assert(WIN_STEPS % SLOT_STEPS == 0 && (NSLOT * SLOT_STEPS) % WIN_STEPS == 0,
              "a window's K-steps occupy whole slots");
static_assert(SMEM_ALLOC <= 232448, "shared memory per block");
static_assert(TM * KS / 8 == SPLIT_THREADS, "items of a block");
static_assert(NFOLD % 128 == 0, "fold warp w covers TMEM lane quarter w % 4");

__device__ __forceinline__ uint64_t wait_ns(bool expired) {
  return expired ? 1000000ull : WAIT_TIMEOUT_NS;
}

// Byte offset, inside one part, of the 16-byte core-matrix row holding elements (r, 8 kc ..
// 8 kc + 7) of a block -- r the M (or N) index in the tile, kc the 8-element chunk of the K-step:
// K-major core matrices (8 rows x 16 bytes), LBO 128 (the two chunks along K), SBO 256 (8-row
// groups).
__device__ __forceinline__ uint32_t kc_off(int r, int kc) {
  return static_cast<uint32_t>(((r >> 3) << 8) + (kc << 7) + ((r & 7) << 4));
}

// ---------------------------------------------------------------------------------------------
// The split: each operand, once per product, into bf16 parts in the layout the MMA reads.
// ---------------------------------------------------------------------------------------------

// Block (tile t, K-step s) of operand X (A: M x K, or B read as N x K): three parts of [128 rows
// x 16 K] K-major core matrices, 12 KB, at parts + (t * nks + s) * BLOCK. Rows past the
// operand's M (N) and K past its K are zero. One CUDA block per operand block; thread `it` owns
// one 8-element item:
//  - K contiguous (k_contig): row it / 2, elements 8 (it % 2) .. + 7 -- two 16-byte loads when the
//    rows are 16-byte aligned (vec), else eight scalar loads;
//  - otherwise: row it % 128 (a warp: 32 consecutive rows, one coalesced load per K index),
//    elements 8 (it / 128) .. + 7.
// The parts of the item go to the three parts' kc_off(row, chunk): a warp writes 4 x 128 bytes
// contiguous per part.
__global__ void __launch_bounds__(SPLIT_THREADS) linear_split_kernel(const LinArgs a) {
  griddep_wait();  // A and B may come from the previous kernel on the stream
  griddep_launch_dependents();
  const int blocks_a = a.tiles_m * a.nks;
  const bool is_a = static_cast<int>(blockIdx.x) < blocks_a;
  const int blk = is_a ? blockIdx.x : blockIdx.x - blocks_a;
  const int t = blk / a.nks, s = blk % a.nks;
  const float* src = is_a ? a.a : a.b;
  const int64_t s_mn = is_a ? a.a_sm : a.b_sn;
  const int64_t s_k = is_a ? a.a_sk : a.b_sk;
  const int extent = is_a ? a.M : a.N;
  const bool k_contig = is_a ? a.a_k_contig : a.b_k_contig;
  const bool vec = is_a ? a.a_vec : a.b_vec;
  unsigned char* dst = (is_a ? a.pa : a.pb) + static_cast<int64_t>(blk) * BLOCK;
  const int it = threadIdx.x;
  const int r = k_contig ? it >> 1 : it & 127;
  const int kc = k_contig ? it & 1 : it >> 7;
  const int mn = t * TM + r, k0 = s * KS + 8 * kc;
  float x[8];
  if (mn < extent && k_contig && vec && k0 + 8 <= a.K) {
    const float* p = src + static_cast<int64_t>(mn) * s_mn + k0;
    const float4 u = __ldg(reinterpret_cast<const float4*>(p));
    const float4 v = __ldg(reinterpret_cast<const float4*>(p) + 1);
    x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = v.x, x[5] = v.y, x[6] = v.z, x[7] = v.w;
  } else {
    const float* p = src + static_cast<int64_t>(mn) * s_mn;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      x[j] = mn < extent && k0 + j < a.K ? __ldg(p + static_cast<int64_t>(k0 + j) * s_k) : 0.f;
  }
  uint4 p0, p1, p2;
  tc::split8(x, p0, p1, p2);
  const uint32_t off = kc_off(r, kc);
  *reinterpret_cast<uint4*>(dst + off) = p0;
  *reinterpret_cast<uint4*>(dst + PART + off) = p1;
  *reinterpret_cast<uint4*>(dst + 2 * PART + off) = p2;
}

// ---------------------------------------------------------------------------------------------
// The product: bulk copies of the parts, six MMAs a K-step, fp32 folds a window.
// ---------------------------------------------------------------------------------------------

// The six products of each of a slot's two K-steps (A's parts of K-step t at descriptor words
// a_lo + 768 t + 256 i, B's at b_lo + 768 t + 256 j: parts PART bytes, blocks BLOCK bytes apart):
// the five small ones into `lo`, A0B0 into `hi`. acc = 0 starts both accumulators afresh (the
// slot opens a window). Two asm blocks for the warp, each with one elect.sync and immediate
// offsets: the first ten MMAs, then (issue_slot_tail) the last two -- the MMA warp waits for the
// next slot between them, while the tensor core still has queued work.
#define LMMA(D, AO, BO, P)                                                  \
  "add.u32 al, %2, " #AO ";\n\t"                                            \
  "add.u32 bl, %4, " #BO ";\n\t"                                            \
  "mov.b64 ad, {al, %3};\n\t"                                               \
  "mov.b64 bd, {bl, %5};\n\t"                                               \
  "@e tcgen05.mma.cta_group::1.kind::f16 [" D "], ad, bd, %6, " #P ";\n\t"
#define LMMA_BEGIN                                                          \
  "{\n\t.reg .pred e, pa, pt;\n\t.reg .b32 al, bl;\n\t.reg .b64 ad, bd;\n\t"   \
  "elect.sync _|e, 0xffffffff;\n\t"                                         \
  "setp.ne.b32 pa, %7, 0;\n\tsetp.eq.b32 pt, %7, %7;\n\t"
static_assert(PART >> 4 == 256 && BLOCK >> 4 == 768 && SLOT_STEPS == 2, "descriptor offsets");
__device__ __forceinline__ void issue_slot_head(uint32_t d_hi, uint32_t d_lo, uint32_t a_lo,
                                                uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                                uint32_t idesc, uint32_t acc) {
  asm volatile(LMMA_BEGIN
      LMMA("%1", 0, 256, pa)
      LMMA("%1", 256, 0, pt)
      LMMA("%1", 0, 512, pt)
      LMMA("%1", 256, 256, pt)
      LMMA("%1", 512, 0, pt)
      LMMA("%0", 0, 0, pa)
      LMMA("%1", 768, 1024, pt)
      LMMA("%1", 1024, 768, pt)
      LMMA("%1", 768, 1280, pt)
      LMMA("%1", 1024, 1024, pt)
      "}\n" ::"r"(d_hi), "r"(d_lo), "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc),
      "r"(acc)
      : "memory");
}
__device__ __forceinline__ void issue_slot_tail(uint32_t d_hi, uint32_t d_lo, uint32_t a_lo,
                                                uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                                uint32_t idesc) {
  asm volatile(LMMA_BEGIN
      LMMA("%1", 1280, 768, pt)
      LMMA("%0", 768, 768, pt)
      "}\n" ::"r"(d_hi), "r"(d_lo), "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc),
      "r"(1u)
      : "memory");
}
#undef LMMA
#undef LMMA_BEGIN

__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Item li of this block: its output tile's row and column tiles and its K chunk. Consecutive
// items share A's row panel.
__device__ __forceinline__ void item_geom(const LinArgs& a, int li, int& tm, int& tn,
                                          int& chunk) {
  const int tiles = a.tiles_m * a.tiles_n;
  const int it = static_cast<int>(blockIdx.x) + li * static_cast<int>(gridDim.x);
  const int tile = it % tiles;
  chunk = it / tiles;
  tm = tile / a.tiles_n;
  tn = tile % a.tiles_n;
}

__global__ void __launch_bounds__(NTHR, 1) linear_tc_kernel(const LinArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* sm = smem_raw + ((128u - (raw & 127u)) & 127u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + OFF_BAR);  // [NSLOT]: the slot's parts landed
  uint64_t* empty = full + NSLOT;     // [NSLOT]: the slot's MMAs completed
  uint64_t* accf = full + 2 * NSLOT;  // [2]: the window's products completed
  uint64_t* acce = accf + 2;          // [2]: the window's sums read (one arrival per fold warp)
  uint32_t* tbase_p = reinterpret_cast<uint32_t*>(full + NBAR);

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < NSLOT; ++i) {
      tc::mbar_init(full + i, 1);
      tc::mbar_init(empty + i, 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(accf + i, 1);
      tc::mbar_init(acce + i, NFOLD / 32);
    }
    tc::fence_mbar_init();
  }
  griddep_wait();  // the parts come from the split kernel before this one
  griddep_launch_dependents();
  __syncthreads();
  if (w == MMA_WARP) {
    tc::tmem_alloc(tbase_p, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tbase_p;

  const int G = static_cast<int>(gridDim.x);
  const int my_items = (a.n_items - static_cast<int>(blockIdx.x) + G - 1) / G;
  const int total = my_items * a.chunk_steps;  // K-steps of this block, a multiple of WIN_STEPS
  bool err = false;

  if (w == PRODUCER_WARP) {
    // ---- producer: one lane, two bulk copies a K-step into the ring ----
    if (lane == 0) {
      const unsigned char* pa = nullptr;
      const unsigned char* pb = nullptr;
      int left = 0, li = 0;
      for (int g = 0; g < total / SLOT_STEPS; ++g) {  // g: slot use
        if (left == 0) {  // the block's next item
          int tm, tn, chunk;
          item_geom(a, li++, tm, tn, chunk);
          const int64_t k0 = static_cast<int64_t>(chunk) * a.chunk_steps;
          pa = a.pa + (static_cast<int64_t>(tm) * a.nks + k0) * BLOCK;
          pb = a.pb + (static_cast<int64_t>(tn) * a.nks + k0) * BLOCK;
          left = a.chunk_steps / SLOT_STEPS;
        }
        const int slot = g % NSLOT;
        if (g >= NSLOT) err |= !tc::mbar_wait(empty + slot, ((g / NSLOT) - 1) & 1, wait_ns(err));
        unsigned char* dst = sm + slot * SLOT;
        tc::mbar_arrive_expect_tx(full + slot, SLOT);
        tc::bulk_load(dst, pa, SLOT_STEPS * BLOCK, full + slot);
        tc::bulk_load(dst + SLOT_STEPS * BLOCK, pb, SLOT_STEPS * BLOCK, full + slot);
        pa += SLOT_STEPS * BLOCK;
        pb += SLOT_STEPS * BLOCK;
        --left;
      }
    }
    __syncwarp();
  } else if (w == MMA_WARP) {
    // ---- MMA warp ----
    const uint32_t idesc = tc::idesc_f32acc(1, TM, TN);
    const uint32_t s0 = tc::smem_u32(sm);
    const tc::Desc ad = tc::split_desc(tc::desc_kmajor(s0, 128, 256));
    const tc::Desc bd = tc::split_desc(tc::desc_kmajor(s0 + SLOT_STEPS * BLOCK, 128, 256));
    constexpr int SLOTS_PER_WIN = WIN_STEPS / SLOT_STEPS;
    const int uses = total / SLOT_STEPS;
    // Slot use g's operands in place (and, when g opens window wl >= 2, the fold warps done with
    // window wl - 2's accumulator pair).
    auto wait_use = [&](int g) {
      const int wl = g / SLOTS_PER_WIN;
      if (g % SLOTS_PER_WIN == 0 && wl >= 2)
        err |= !tc::mbar_wait(acce + (wl & 1), ((wl >> 1) - 1) & 1, wait_ns(err));
      err |= !tc::mbar_wait(full + g % NSLOT, (g / NSLOT) & 1, wait_ns(err));
      tc::fence_after_sync();
    };
    wait_use(0);
    for (int g = 0; g < uses; ++g) {  // g: slot use
      const int js = g % SLOTS_PER_WIN, wl = g / SLOTS_PER_WIN, b = wl & 1;
      const int slot = g % NSLOT;
      const uint32_t so = static_cast<uint32_t>(slot * (SLOT >> 4));
      const uint32_t d_hi = tbase + 256u * b, d_lo = d_hi + 128u;
      const uint32_t a_lo = tc::opaque(ad.lo + so), b_lo = tc::opaque(bd.lo + so);
      issue_slot_head(d_hi, d_lo, a_lo, ad.hi, b_lo, bd.hi, idesc, js != 0);
      if (g + 1 < uses) wait_use(g + 1);
      issue_slot_tail(d_hi, d_lo, a_lo, ad.hi, b_lo, bd.hi, idesc);
      tc::commit_warp(empty + slot);
      if (js == SLOTS_PER_WIN - 1) tc::commit_warp(accf + b);
    }
  } else {
    // ---- fold warps: thread (lane quarter q, column half h) owns row 32 q + lane, columns
    // FC h .. + FC - 1 of the tile ----
    const int q = w & 3, half = w >> 2;
    const uint32_t lane_sel = static_cast<uint32_t>(32 * q) << 16;
    const int wins_per_item = a.chunk_steps / WIN_STEPS;
    uint64_t acc[FC / 2];  // columns FC half + 2 i, + 1 (packed pairs)
#pragma unroll
    for (int i = 0; i < FC / 2; ++i) acc[i] = 0;
    for (int wl = 0; wl < total / WIN_STEPS; ++wl) {
      const int b = wl & 1;
      err |= !tc::mbar_wait(accf + b, (wl >> 1) & 1, wait_ns(err));
      tc::fence_after_sync();
      const uint32_t t_hi = tbase + lane_sel + 256u * b + static_cast<uint32_t>(FC * half);
#pragma unroll
      for (int j = 0; j < FC / 16; ++j) {
        float hi[16], lo[16];
        tc::tmem_ld16(t_hi + 16 * j, hi);
        tc::tmem_ld16(t_hi + 128 + 16 * j, lo);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          acc[8 * j + i] = add2(acc[8 * j + i], add2(tc::pack2(hi[2 * i], hi[2 * i + 1]),
                                                     tc::pack2(lo[2 * i], lo[2 * i + 1])));
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acce + b);
      if ((wl + 1) % wins_per_item == 0) {
        int tm, tn, chunk;
        item_geom(a, wl / wins_per_item, tm, tn, chunk);
        const int nb = tn * TN + FC * half;
        if (!err) {
          // The output (one chunk: C; several: this chunk's partial tile, rows ldp apart), 32
          // columns at a time through this warp's staging block: each lane writes its row's 32
          // floats (16-byte chunk c of row r at chunk c ^ (r % 8): no bank conflict), then the
          // warp writes four whole 128-byte rows per instruction.
          float* const out_rows = a.ksplit == 1 ? a.c : a.part + static_cast<int64_t>(chunk) * a.M * a.ldp;
          const int64_t ld = a.ksplit == 1 ? a.c_sm : a.ldp;
          const int n_end = a.ksplit == 1 ? a.N : a.ldp;
          float4* stage = reinterpret_cast<float4*>(sm + OFF_OUT + w * OUT_WARP);
          const int m0 = tm * TM + 32 * q;  // the warp's first row
#pragma unroll
          for (int h2 = 0; h2 < FC / 32; ++h2) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              float x0, x1, x2, x3;
              tc::unpack2(acc[16 * h2 + 2 * c], x0, x1);
              tc::unpack2(acc[16 * h2 + 2 * c + 1], x2, x3);
              stage[lane * 8 + (c ^ (lane & 7))] = make_float4(x0, x1, x2, x3);
            }
            __syncwarp();
            const int c = lane & 7;
            const int n = nb + 32 * h2 + 4 * c;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 4 * i + (lane >> 3);
              const float4 v = stage[r * 8 + (c ^ (r & 7))];
              const int m = m0 + r;
              if (m < a.M) {
                float* dst = out_rows + static_cast<int64_t>(m) * ld + n;
                if (n + 4 <= n_end) {
                  *reinterpret_cast<float4*>(dst) = v;
                } else if (n < n_end) {
                  dst[0] = v.x;
                  if (n + 1 < n_end) dst[1] = v.y;
                  if (n + 2 < n_end) dst[2] = v.z;
                }
              }
            }
            __syncwarp();
          }
        }
#pragma unroll
        for (int i = 0; i < FC / 2; ++i) acc[i] = 0;
      }
    }
  }

  if (__syncthreads_or(err)) {
    if (tid == 0) {
      atomicExch(&g_linear_err, 1);
      flag_timeout(nullptr, a.sink);
    }
    // The last window's commit covers every MMA of the block: one more bounded wait for it.
    if (w == MMA_WARP && total > 0) {
      const int wl = total / WIN_STEPS - 1;
      tc::mbar_wait(accf + (wl & 1), (wl >> 1) & 1, WAIT_TIMEOUT_NS);
    }
    // The producer's last copies complete on their slots' full barriers.
    if (w == PRODUCER_WARP && lane == 0) {
      const int uses = total / SLOT_STEPS;
      for (int g = max(0, uses - NSLOT); g < uses; ++g)
        tc::mbar_wait(full + g % NSLOT, (g / NSLOT) & 1, WAIT_TIMEOUT_NS);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (w == MMA_WARP) tc::tmem_dealloc(tbase, TMEM_COLS);
}

// C = sum of the K chunks' partial tiles, in chunk order (float4 columns; ldp % 4 == 0).
__global__ void __launch_bounds__(256) linear_reduce_kernel(const LinArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int q4 = a.ldp / 4;
  const int64_t n4 = static_cast<int64_t>(a.M) * q4;
  const int64_t plane = static_cast<int64_t>(a.M) * a.ldp;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / q4), n = 4 * static_cast<int>(i % q4);
    if (n >= a.N) continue;
    const float* p = a.part + static_cast<int64_t>(m) * a.ldp + n;
    float4 s = *reinterpret_cast<const float4*>(p);
    for (int ch = 1; ch < a.ksplit; ++ch) {
      const float4 t = *reinterpret_cast<const float4*>(p + ch * plane);
      s.x += t.x, s.y += t.y, s.z += t.z, s.w += t.w;
    }
    float* dst = a.c + static_cast<int64_t>(m) * a.c_sm + n;
    if (n + 4 <= a.N) {
      *reinterpret_cast<float4*>(dst) = s;
    } else {
      dst[0] = s.x;
      if (n + 1 < a.N) dst[1] = s.y;
      if (n + 2 < a.N) dst[2] = s.z;
    }
  }
}

// C = 0 (an empty reduction, K = 0), row by row.
__global__ void __launch_bounds__(256) linear_zero_kernel(const LinArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t n = static_cast<int64_t>(a.M) * a.N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    a.c[(i / a.N) * a.c_sm + i % a.N] = 0.f;
}


}  // namespace

LinPlan linear_plan(int64_t M, int64_t N, int64_t K) {
  LinPlan p{};
  p.tiles_m = static_cast<int>((M + TM - 1) / TM);
  p.tiles_n = static_cast<int>((N + TN - 1) / TN);
  const int64_t kwin = (K + KS * WIN_STEPS - 1) / (KS * WIN_STEPS);
  const int64_t tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  // K chunks: enough items for the B200's 148 SMs when the output alone has fewer tiles, at least
  // 4 windows a chunk. A function of the shape only (never of the device), so the summation order
  // -- and the bits -- are the same on every GPU.
  int64_t ks = tiles >= LIN_SMS ? 1 : std::max<int64_t>(1, LIN_SMS / std::max<int64_t>(tiles, 1));
  ks = std::min<int64_t>(ks, std::max<int64_t>(1, kwin / 4));
  const int64_t cw = (kwin + ks - 1) / ks;  // windows per chunk
  p.ksplit = static_cast<int>((kwin + cw - 1) / cw);
  p.chunk_steps = static_cast<int>(cw * WIN_STEPS);
  p.ldp = static_cast<int>((N + 3) / 4 * 4);
  p.nks = p.ksplit * p.chunk_steps;
  const size_t pa = static_cast<size_t>(p.tiles_m) * p.nks * BLOCK;
  const size_t pb = static_cast<size_t>(p.tiles_n) * p.nks * BLOCK;
  const size_t part = p.ksplit > 1 ? static_cast<size_t>(p.ksplit) * M * p.ldp * sizeof(float) : 0;
  p.pa_off = 0;
  p.pb_off = align256(pa);
  p.part_off = p.pb_off + align256(pb);
  p.ws_bytes = p.part_off + align256(part);
  return p;
}

cudaError_t setup_linear_attributes() {
  return cudaFuncSetAttribute(linear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              SMEM_ALLOC);
}

cudaError_t launch_linear_tc(const LinArgs& args, cudaStream_t stream) {
  LinArgs a = args;
  if (a.K == 0) {
    const int64_t n = static_cast<int64_t>(a.M) * a.N;
    const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4096));
    return launch_pdl(linear_zero_kernel, dim3(blocks), dim3(256), 0, stream, a);
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = LIN_SMS;
  a.n_items = a.tiles_m * a.tiles_n * a.ksplit;
  const dim3 split_grid(static_cast<unsigned>((a.tiles_m + a.tiles_n) * a.nks));
  cudaError_t e = launch_pdl(linear_split_kernel, split_grid, dim3(SPLIT_THREADS), 0, stream, a);
  if (e != cudaSuccess) return e;
  const dim3 grid(static_cast<unsigned>(std::min(a.n_items, sms)));
  e = launch_pdl(linear_tc_kernel, grid, dim3(NTHR), SMEM_ALLOC, stream, a);
  if (e != cudaSuccess || a.ksplit == 1) return e;
  const int64_t n4 = static_cast<int64_t>(a.M) * (a.ldp / 4);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n4 + 255) / 256, 4 * sms));
  return launch_pdl(linear_reduce_kernel, dim3(blocks), dim3(256), 0, stream, a);
}

cudaError_t linear_status(int* flag) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_linear_err, sizeof(int));
  if (e != cudaSuccess) return e;
  *flag = v;
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_linear_err, &zero, sizeof(int));
  }
  return e;
}

}  // namespace cfa
