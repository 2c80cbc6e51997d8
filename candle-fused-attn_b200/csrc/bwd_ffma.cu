// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The backward: dQ, dK, dV of O = softmax(Q K^T * scale) V from dO, the forward's O and its row
// log-sum-exp L, written into ONE [b, s, 3, h, 64] buffer (a fused qkv projection's gradient).
// Replaces fattn_bwd_dot_f32_d64 and fattn_bwd_f32_d64 (kernels/fused_attn.cu:45-63, :213-426).
//
// Step 1 (prep kernel): D[b, h, i] = sum_d dO[i, d] O[i, d] in fp64, 16 lanes per row, one float4
// each, then the 16-lane butterfly, rounded once to fp32; the same kernel clears the work ticket, the error flag and the dQ
// turn counters that step 2 uses (the stream orders it before step 2).
//
// Step 2 (main kernel): one block per key block of BWD_BN = 64 keys of one (batch, head); K and
// V stay in shared memory, dK and dV in registers. The block walks query tiles of BWD_BM = 64:
//   phase 1: warps 0-3 compute S = Q K^T and P = exp(S * scale - L) (masked), warps 4-7 compute
//            dP = dO V^T; each thread an 8 x 4 tile (rows 16(w%4) + ty + 2i, keys tx + 16jj).
//            Then warps 4-7 form dS = P o (dP - D) at the same positions.
//   phase 2: warps 0-3 accumulate dV += P^T dO, warps 4-7 dK += dS^T Q; each thread 8 keys x 4
//            dims (keys 16(w%4) + 8ty .. +8, dims 4tx .. +4), summed over the tile's queries in
//            index order.
//   phase 3: all warps compute the tile's dQ partial dS K (rows 8w + ty + 2i, dims 4tx .. +4)
//            and add it into dQ in KEY-BLOCK ORDER: key block 0 stores, each later one reads
//            (through L2), adds and stores, the last contributor multiplies by `scale`. A turn
//            counter per (batch, head, query tile) hands the tile from one key block to the next.
//   Five products per tile, S and dP computed once (the reference's split: kernels/fused_attn.cu
//   :178-205), no atomics on data: dQ = ((p0 + p1) + p2) + ... for every schedule.
//
// Forward progress without dispatch-order assumptions: a block takes its (batch, head, key block)
// from a global ticket (atomicAdd), key-block-major, so a block only ever waits on blocks holding
// smaller tickets, which are already running or done.
// Every wait is bounded (cfa::WAIT_TIMEOUT_NS); on expiry the error flag is set and the host
// reads it with cfa_bwd_status. No GPU hangs on a broken invariant.
#include "cfa_common.cuh"

namespace cfa {
namespace {

constexpr int BWD_SMEM_FLOATS = 4 * 64 * LD + 2 * 64 * LDP + 2 * 64 + 4;

__global__ void __launch_bounds__(PREP_THREADS) bwd_prep_kernel(const PrepArgs a) {
  griddep_wait();  // O (the forward's) and dO may come from the previous kernel
  griddep_launch_dependents();
  const int64_t gtid = static_cast<int64_t>(blockIdx.x) * PREP_THREADS + threadIdx.x;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * PREP_THREADS;
  for (int64_t z = gtid; z < a.n_zero; z += gstride) a.zero[z] = 0;

  const int64_t rows = static_cast<int64_t>(a.B) * a.H * a.S;
  const int64_t row = gtid >> 4;  // row = (b * H + h) * S + i
  const int c = threadIdx.x & 15;
  double x = 0.0;
  if (row < rows) {
    const int i = static_cast<int>(row % a.S);
    const int64_t bhr = row / a.S;
    const int h = static_cast<int>(bhr % a.H), b = static_cast<int>(bhr / a.H);
    const float4 ov = ld4(a.o + ((static_cast<int64_t>(b) * a.S + i) * a.H + h) * 64 + 4 * c);
    const float4 gv = ld4(a.d_o + b * a.do_sb + h * a.do_sh + i * a.do_ss + 4 * c);
    // In fp64 (the kernel is bound by HBM, not arithmetic): D feeds the cancellation dP - D of
    // every dS, so its error matters more than one product's. Products of two floats are exact
    // in fp64.
    x = __fma_rn(static_cast<double>(ov.w), gv.w,
            __fma_rn(static_cast<double>(ov.z), gv.z,
                __fma_rn(static_cast<double>(ov.y), gv.y, static_cast<double>(ov.x) * gv.x)));
  }
  // DETERMINISM: four products per lane in d order, then the butterfly 1, 2, 4, 8.
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  if (row < rows && c == 0) a.dsum[row] = static_cast<float>(x);
}

// Phase 1 products for this thread's 8 rows (rb1 + 2i) and the first JN of its 4 key groups
// (keys tx + 16jj): s = A B^T over d as an even-d chain plus an odd-d chain (packed FMAs), the
// same order as the forward's scores. Rows in two halves of 4 (32 packed accumulators live).
// Key groups jj >= JN lie wholly past the sequence end: left at 0 (masked or multiplied by P = 0).
template <int JN>
__device__ __forceinline__ void phase1_tile(const float* As, const float* Bs, int rb1, int tx,
                                            float (&s)[8][4]) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    uint64_t s2[4][JN];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < JN; ++jj) s2[i][jj] = 0ull;
#pragma unroll 2
    for (int c = 0; c < 64; c += 4) {
      ulonglong2 bv[JN], av[4];
#pragma unroll
      for (int jj = 0; jj < JN; ++jj) bv[jj] = ld2x2(Bs + (tx + 16 * jj) * LD + c);
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = ld2x2(As + (rb1 + 2 * (4 * hh + i)) * LD + c);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < JN; ++jj) s2[i][jj] = fma2(av[i].x, bv[jj].x, s2[i][jj]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < JN; ++jj) s2[i][jj] = fma2(av[i].y, bv[jj].y, s2[i][jj]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        s[4 * hh + i][jj] = jj < JN ? sum2(s2[i][jj < JN ? jj : 0]) : 0.0f;
  }
}

template <bool CAUSAL>
__global__ void __launch_bounds__(BWD_THREADS, 2) bwd_ffma_kernel(const BwdArgs a) {
  extern __shared__ float4 smem4[];
  float* Ks = reinterpret_cast<float*>(smem4);  // [64][LD]
  float* Vs = Ks + 64 * LD;                     // [64][LD]
  float* Qs = Vs + 64 * LD;                     // [64][LD]
  float* dOs = Qs + 64 * LD;                    // [64][LD]
  float* Ps = dOs + 64 * LD;                    // [64][LDP] query-major
  float* dSs = Ps + 64 * LDP;                   // [64][LDP] query-major
  float* Lt = dSs + 64 * LDP;                   // [64] L of this tile (0 past S)
  float* Dt = Lt + 64;                          // [64] D of this tile (0 past S)
  int* s_int = reinterpret_cast<int*>(Dt + 64); // [0]: ticket, [1]: turn came

  griddep_launch_dependents();
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int ty = lane >> 4, tx = lane & 15;
  const int grp = w >> 2, wg = w & 3;  // grp 0: S, P, dV; grp 1: dP, dS, dK (warp-uniform)
  const int S = a.S;

  // The prep kernel's writes (D, the cleared ticket and counters) are awaited before their first
  // use. The no-wait path (dQ partials) never waits on another block: its block index is its
  // ticket, and the block's first tiles of q, k, v, dO -- inputs no kernel of this chain writes,
  // read through L2 only -- load while the prep kernel finishes. The turn chain draws tickets
  // (forward progress, below).
  const bool no_wait = a.dq_part != nullptr;
  int ticket;
  if (no_wait) {
    ticket = static_cast<int>(blockIdx.x);
  } else {
    griddep_wait();
    if (tid == 0) s_int[0] = atomicAdd(a.ticket, 1);
    __syncthreads();
    ticket = s_int[0];
  }
  // Tickets run key-block-major: every (b, h) of key block 0, then of key block 1, ... A block of
  // the turn chain waits only on key block kb - 1 of its (b, h), which holds a smaller ticket, so
  // it is running or done; and blocks of similar length (causal: block kb walks n_qtiles - kb
  // tiles) share a wave, longest first, instead of a wave holding every key block of one (b, h)
  // that all end with its key block 0.
  const int BH = a.B * a.H;
  // (Non-causal, no-wait path: (b, h)-major instead, so each (b, h)'s last block -- the one that
  // sums its dQ partials -- finishes throughout the run rather than all in the last wave.)
  const bool bh_major = !CAUSAL && no_wait;
  const int kb = bh_major ? ticket % a.n_kblocks : ticket / BH;
  const int bh = bh_major ? ticket / a.n_kblocks : ticket % BH;
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kb * BWD_BN;

  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* gp = a.d_o + b * a.do_sb + h * a.do_sh;
  const float* lp = a.lse + static_cast<int64_t>(bh) * S;
  const float* dp = a.dsum + static_cast<int64_t>(bh) * S;
  int* turn = a.turn + static_cast<int64_t>(bh) * a.n_qtiles;
  const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * 64;  // dqkv floats per (b, s)
  float* dq_base = a.dqkv + static_cast<int64_t>(b) * S * row_stride + h * 64;

  load_tile_async<64, BWD_THREADS>(Ks, a.k + b * a.k_sb + h * a.k_sh, a.k_ss, k0, S);
  load_tile_async<64, BWD_THREADS>(Vs, a.v + b * a.v_sb + h * a.v_sh, a.v_ss, k0, S);

  // grp 0: dV, grp 1: dK (unscaled): acc2[rp][e] holds keys 16wg + 8ty + 2rp and + 2rp + 1 (the
  // two halves of the pair), dim 4tx + e.
  uint64_t acc2[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc2[i][e] = 0ull;

  const int rb1 = 16 * wg + ty;       // phase 1 rows: rb1 + 2i
  const int kb2 = 16 * wg + 8 * ty;   // phase 2 keys: kb2 .. kb2 + 7
  const int rb3 = 8 * w + ty;         // phase 3 rows: rb3 + 2i

  // Q, dO, then L, D of query tile q0 into the (single) tile buffers; one cp.async group.
  auto load_q_do = [&](int q0) {
    load_tile_async<64, BWD_THREADS>(Qs, qp, a.q_ss, q0, S);
    load_tile_async<64, BWD_THREADS>(dOs, gp, a.do_ss, q0, S);
  };
  auto load_l_d = [&](int q0) {
    if (tid < 128) {
      const int r = tid & 63, i = q0 + r;
      const bool ok = i < S;
      const float* src = (tid < 64 ? lp : dp) + (ok ? i : q0);
      cp_async4((tid < 64 ? Lt : Dt) + r, src, ok ? 4 : 0);
    }
  };
  auto load_query_tile = [&](int q0) {
    load_q_do(q0);
    load_l_d(q0);
  };

  // Causal: queries before the block's first key never see it.
  const int t_begin = CAUSAL ? k0 / BWD_BM : 0;
  load_q_do(t_begin * BWD_BM);
  if (no_wait) griddep_wait();
  load_l_d(t_begin * BWD_BM);
  cp_async_commit();
  for (int t = t_begin; t < a.n_qtiles; ++t) {
    const int q0 = t * BWD_BM;
    // This tile (and the first time K, V) has landed, and every thread is done with the previous
    // tile (its dS reads of phase 3 included).
    cp_async_wait_all();
    __syncthreads();

    // Dead work on edge tiles is skipped, uniformly per tile: key groups wholly past the sequence
    // end (jn) and query rows past it in the phase-2 sums (iq); and, uniformly per warp, a warp
    // whose rows (phases 1 and 3) or keys (phase 2) all lie past the end does no products. The
    // skipped terms are masked scores and products with P = 0 or dS = 0: the live results are
    // the same bits either way. (Canvas s = 240: -2.7% time; the forward's counterpart measured
    // slower and is not done.)
    const int jn = min(4, (S - k0 + 15) / 16);
    const int iq = min(BWD_BM, (S - q0 + 15) / 16 * 16);

    // Phase 1. grp 0: s = Q K^T; grp 1: s = dO V^T (dP), as even/odd packed chains.
    {
      const float* As = grp ? dOs : Qs;
      const float* Bs = grp ? Vs : Ks;
      float s[8][4];
      if (q0 + 16 * wg >= S) {
        // rows 16 wg .. 16 wg + 15 all past the end: s = 0 gives P = 0 (masked) and dS = 0
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) s[i][jj] = 0.0f;
      } else if (jn == 4)
        phase1_tile<4>(As, Bs, rb1, tx, s);
      else if (jn == 3)
        phase1_tile<3>(As, Bs, rb1, tx, s);
      else if (jn == 2)
        phase1_tile<2>(As, Bs, rb1, tx, s);
      else
        phase1_tile<1>(As, Bs, rb1, tx, s);
      if (grp == 0) {
        const bool edge = (q0 + BWD_BM > S) || (k0 + BWD_BN > S) ||
                          (CAUSAL && k0 + BWD_BN - 1 > q0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int il = rb1 + 2 * i, qi = q0 + il;
          const float li = Lt[il];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int jl = tx + 16 * jj, j = k0 + jl;
            // P = e^(s * scale - L): the argument in natural units with one rounding.
            float pr = expf(fmaf(s[i][jj], a.scale, -li));
            if (edge && !(qi < S && j < S && !(CAUSAL && j > qi))) pr = 0.0f;
            Ps[il * LDP + jl] = pr;
          }
        }
      }
      __syncthreads();
      if (grp == 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int il = rb1 + 2 * i;
          const float di = Dt[il];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int jl = tx + 16 * jj;
            dSs[il * LDP + jl] = Ps[il * LDP + jl] * (s[i][jj] - di);
          }
        }
      }
      __syncthreads();
    }

    // Phase 2. grp 0: dV[j] += sum_i P[i][j] dO[i]; grp 1: dK[j] += sum_i dS[i][j] Q[i].
    // Packed FMAs with the accumulators paired along keys: (x[j], x[j + 1]) is a register pair of
    // the float4 read from P / dS, the dO / Q element is broadcast; each lane computes the same
    // fmaf per element as scalar code would.
    // DETERMINISM: each dK, dV element is one thread's register, summed over query tiles and
    // then queries in index order.
    {
      const float* Xs = grp ? dSs : Ps;
      const float* Ys = grp ? Qs : dOs;
      const int iw = k0 + 16 * wg >= S ? 0 : iq;  // keys kb2 .. kb2 + 7 all past the end: none
#pragma unroll 4
      for (int i = 0; i < iw; ++i) {
        const ulonglong2 xa = ld2x2(Xs + i * LDP + kb2), xb = ld2x2(Xs + i * LDP + kb2 + 4);
        const float4 y = ld4(Ys + i * LD + 4 * tx);
        const uint64_t xp[4] = {xa.x, xa.y, xb.x, xb.y};
        const uint64_t yb[4] = {dup2(y.x), dup2(y.y), dup2(y.z), dup2(y.w)};
#pragma unroll
        for (int rp = 0; rp < 4; ++rp)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc2[rp][e] = fma2(xp[rp], yb[e], acc2[rp][e]);
      }
    }
    // Every thread is done with Q, dO, L, D of this tile: the next tile's copies travel during
    // phase 3 and the ordered dQ add.
    __syncthreads();
    if (t + 1 < a.n_qtiles) {
      load_query_tile(q0 + BWD_BM);
      cp_async_commit();
    }

    // Phase 3: the dQ partial pq[r][e] = sum_j dS[rb3 + 2r][j] K[j][4tx + e], keys in order.
    // Packed FMAs, accumulators paired along dims ((e, e + 1) of the float4 read from K), the
    // dS element broadcast: the same fmaf per element as scalar code.
    uint64_t pq2[4][2];
#pragma unroll
    for (int r = 0; r < 4; ++r) pq2[r][0] = pq2[r][1] = 0ull;
    const int jlim = q0 + 8 * w >= S ? 0 : 16 * jn;  // rows rb3 + 2r all past the end: none
#pragma unroll 2
    for (int j = 0; j < jlim; j += 4) {
      ulonglong2 k4[4];
      float4 d4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) k4[u] = ld2x2(Ks + (j + u) * LD + 4 * tx);
#pragma unroll
      for (int r = 0; r < 4; ++r) d4[r] = ld4(dSs + (rb3 + 2 * r) * LDP + j);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint64_t ds = dup2(f4c(d4[r], u));
          pq2[r][0] = fma2(ds, k4[u].x, pq2[r][0]);
          pq2[r][1] = fma2(ds, k4[u].y, pq2[r][1]);
        }
    }
    float pq[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float2 lo = split2(pq2[r][0]), hi = split2(pq2[r][1]);
      pq[r][0] = lo.x;
      pq[r][1] = lo.y;
      pq[r][2] = hi.x;
      pq[r][3] = hi.y;
    }

    if (a.dq_part != nullptr) {
      // No-wait path: this key block's partial for the tile goes to its own scratch rows.
      float* part = a.dq_part + (static_cast<int64_t>(bh) * a.n_kblocks + kb) * S * 64;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int qi = q0 + rb3 + 2 * r;
        if (qi < S)
          __stcg(reinterpret_cast<float4*>(part + static_cast<int64_t>(qi) * 64 + 4 * tx),
                 make_float4(pq[r][0], pq[r][1], pq[r][2], pq[r][3]));
      }
      continue;
    }
    // Turn chain. This tile's contributors are key blocks 0 .. last (causal: those holding a key
    // <= the tile's last query); each adds on its turn.
    const int last = CAUSAL ? min(a.n_kblocks - 1, min(S - 1, q0 + BWD_BM - 1) / BWD_BN)
                            : a.n_kblocks - 1;
    bool go = true;
    if (kb > 0) {
      if (tid == 0) {
        s_int[1] = wait_turn_bounded(turn + t, kb, a.err, a.timeout_ns, a.sink) ? 1 : 0;
        // ORDER: with the barrier below, extends thread 0's acquire to the whole block.
        __threadfence();
      }
      __syncthreads();
      go = s_int[1] != 0;
    }
    if (go) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int qi = q0 + rb3 + 2 * r;
        if (qi >= S) continue;
        float4* dst = reinterpret_cast<float4*>(dq_base + qi * row_stride + 4 * tx);
        float4 v = make_float4(pq[r][0], pq[r][1], pq[r][2], pq[r][3]);
        if (kb > 0) {
          // Through L2 (__ldcg / __stcg): L1 is not coherent across SMs.
          const float4 prev = __ldcg(dst);
          v = make_float4(prev.x + v.x, prev.y + v.y, prev.z + v.z, prev.w + v.w);
        }
        if (kb == last)
          v = make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
        __stcg(dst, v);
      }
    }
    if (kb < last) {
      // ORDER: every thread's dQ stores are visible GPU-wide before thread 0 hands the tile to
      // key block kb + 1 (its acquire in wait_turn_bounded).
      __threadfence();
      __syncthreads();
      if (tid == 0) st_release_gpu(turn + t, kb + 1);
    }
  }

  if (a.dq_part != nullptr) {
    // ORDER: this block's partials are visible GPU-wide before it counts itself in; the block
    // that counts last then reads every partial of its (batch, head).
    __threadfence();
    __syncthreads();
    if (tid == 0) s_int[1] = atomicAdd(a.turn + bh, 1);
    __syncthreads();
    if (s_int[1] == a.n_kblocks - 1) {
      __threadfence();
      const float* part = a.dq_part + static_cast<int64_t>(bh) * a.n_kblocks * S * 64;
      // DETERMINISM: dQ = (((p0 + p1) + p2) + ...) * scale over the contributing key blocks in
      // index order: the turn chain's sums, bit for bit, whichever block does them. Eight rows
      // per thread in flight at once (their partial loads are independent).
      constexpr int R = 8;
      for (int base = 0; base < S * 16; base += BWD_THREADS * R) {
        float4 v[R];
        int last[R];
#pragma unroll
        for (int u = 0; u < R; ++u) {
          const int idx = base + u * BWD_THREADS + tid;
          const int i = min(idx, S * 16 - 1) >> 4, c4 = idx & 15;
          const int t = i / BWD_BM;
          last[u] = CAUSAL
                        ? min(a.n_kblocks - 1, min(S - 1, t * BWD_BM + BWD_BM - 1) / BWD_BN)
                        : a.n_kblocks - 1;
          v[u] = __ldcg(reinterpret_cast<const float4*>(part + static_cast<int64_t>(i) * 64 +
                                                        4 * c4));
        }
        for (int j = 1; j < a.n_kblocks; ++j) {
#pragma unroll
          for (int u = 0; u < R; ++u) {
            const int idx = base + u * BWD_THREADS + tid;
            const int i = min(idx, S * 16 - 1) >> 4, c4 = idx & 15;
            if (j <= last[u]) {
              const float4 p = __ldcg(reinterpret_cast<const float4*>(
                  part + (static_cast<int64_t>(j) * S + i) * 64 + 4 * c4));
              v[u] = make_float4(v[u].x + p.x, v[u].y + p.y, v[u].z + p.z, v[u].w + p.w);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < R; ++u) {
          const int idx = base + u * BWD_THREADS + tid;
          if (idx < S * 16) {
            const int i = idx >> 4, c4 = idx & 15;
            *reinterpret_cast<float4*>(dq_base + i * row_stride + 4 * c4) =
                make_float4(v[u].x * a.scale, v[u].y * a.scale, v[u].z * a.scale,
                            v[u].w * a.scale);
          }
        }
      }
    }
  }

  // grp 0 stores dV into slot 2, grp 1 stores dK * scale into slot 1.
  float* dst0 = a.dqkv + static_cast<int64_t>(b) * S * row_stride + (grp ? 1 : 2) * a.H * 64 +
                h * 64 + 4 * tx;
  const float f = grp ? a.scale : 1.0f;
#pragma unroll
  for (int rp = 0; rp < 4; ++rp) {
    float2 v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = split2(acc2[rp][e]);
    const int j = k0 + kb2 + 2 * rp;
    if (j < S)
      *reinterpret_cast<float4*>(dst0 + j * row_stride) =
          make_float4(v[0].x * f, v[1].x * f, v[2].x * f, v[3].x * f);
    if (j + 1 < S)
      *reinterpret_cast<float4*>(dst0 + (j + 1) * row_stride) =
          make_float4(v[0].y * f, v[1].y * f, v[2].y * f, v[3].y * f);
  }
}

}  // namespace

size_t bwd_smem_bytes() { return BWD_SMEM_FLOATS * sizeof(float); }

cudaError_t setup_bwd_attributes() {
  const int bytes = static_cast<int>(bwd_smem_bytes());
  cudaError_t e = cudaFuncSetAttribute(bwd_ffma_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(bwd_ffma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              bytes);
}

cudaError_t launch_bwd_prep(const PrepArgs& a, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(a.B) * a.H * a.S;
  int64_t blocks = (rows * 16 + PREP_THREADS - 1) / PREP_THREADS;
  if (blocks < 1) blocks = 1;
  return launch_pdl(bwd_prep_kernel, dim3(static_cast<unsigned>(blocks)), dim3(PREP_THREADS), 0,
                    stream, a);
}

cudaError_t launch_bwd(const BwdArgs& a, int causal, cudaStream_t stream) {
  const int64_t blocks = static_cast<int64_t>(a.n_kblocks) * a.B * a.H;
  const dim3 grid(static_cast<unsigned>(blocks));
  if (causal)
    return launch_pdl(bwd_ffma_kernel<true>, grid, dim3(BWD_THREADS), bwd_smem_bytes(), stream, a);
  return launch_pdl(bwd_ffma_kernel<false>, grid, dim3(BWD_THREADS), bwd_smem_bytes(), stream, a);
}

}  // namespace cfa

namespace cfa {
namespace {

// Self-test of the backward's failure detection: every block's thread 0 waits, with the same
// bounded routine the dQ turn chain uses, for a flag that nothing ever sets. Block 0 gives up after
// `short_ns`; the others would wait 100x longer but bail out as soon as block 0 has flagged the
// error. The kernel always ends: with CFA_ERR_TIMEOUT in ws[1] after about `short_ns`.
__global__ void selftest_wait_kernel(int* ws, uint64_t short_ns, int* sink) {
  if (threadIdx.x != 0) return;
  const int* never = ws + 2;  // cleared by the host-side memset; nothing writes it afterwards
  const uint64_t limit = blockIdx.x == 0 ? short_ns : 100 * short_ns;
  wait_turn_bounded(never, 1, ws + 1, limit, sink);
}

}  // namespace

cudaError_t launch_selftest_wait(int* ws, uint64_t short_ns, int blocks, int* sink,
                                 cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(ws, 0, 16, stream);
  if (e != cudaSuccess) return e;
  selftest_wait_kernel<<<blocks, 32, 0, stream>>>(ws, short_ns, sink);
  return cudaGetLastError();
}

}  // namespace cfa
