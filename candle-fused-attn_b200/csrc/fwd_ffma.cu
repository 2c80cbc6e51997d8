// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The forward: O = softmax(Q K^T * scale [+ causal mask]) V over fp32, head_dim 64, with the
// online softmax of FlashAttention-2 (Dao 2023), saving only O and the row log-sum-exp L.
// Replaces fattn_fwd_f32_d64 (kernels/fused_attn.cu:469-598); same inputs, outputs, layouts.
//
// Block: FWD_THREADS = 128 threads (4 warps) own BM = 8 * RPT queries of one (batch, head) and walk
// key tiles of FWD_BN = 64; RPT (rows per thread) is 8 (BM = 64) or 6 (BM = 48), whichever leaves
// fewer padded query rows at the sequence length (fwd_tile_rows). Warp w owns query rows
// 2 RPT w .. 2 RPT w + 2 RPT - 1; within it, lane (ty, tx) = (lane / 16, lane % 16) owns rows
// 2 RPT w + ty + 2i (i < RPT) and
//   - scores for keys tx + 16jj (jj = 0..3): an RPT x 4 register tile, so the row max / sum of the
//     online softmax is a 16-lane butterfly inside one half-warp;
//   - output dims 4tx .. 4tx + 3 of the same 8 rows: the rescale by exp(m_old - m_new) and the
//     final 1 / l never leave the thread.
// Each k-step of 4 reads RPT float4 of Q and 4 of K from shared memory for 16 RPT FFMA (and the
// same for P V), against the reference's 8 loads per 16 FFMA: the FFMA pipe, not the shared-memory
// pipe, is the bound. Three blocks per SM (72.7 / 63.2 KB shared memory, <= 168 registers).
// Rows are independent, so the tile height changes no result bit; it only removes padded rows and
// evens the waves (canvas s = 240: BM = 48, no padded rows, 162.5 -> 148.6 us).
//
// Loads: cp.async (16 B, L2-only) into padded tiles. V(n) travels while S(n) is computed, K(n+1)
// while P V(n) is; Q once. Tiles past `seq` are zero-filled.
//
// DETERMINISM: every sum has one order fixed by the code alone: S over d = 0..63; the row max /
// sum by the butterfly 1, 2, 4, 8; l and O over key tiles in index order, keys 0..63 within one.
#include "cfa_common.cuh"

namespace cfa {
namespace {

template <int RPT>
constexpr int fwd_smem_floats() {
  return (8 * RPT + 2 * FWD_BN) * LD + 8 * RPT * LDP;
}

// S = Q K^T for this thread's NR rows (rb + 2i) and the first JN of its 4 key groups (keys
// tx + 16jj), with packed FMAs: each score is an even-d chain plus an odd-d chain (a float4 of Q
// and one of K give the pairs (d, d + 1), (d + 2, d + 3) directly), each in increasing d, added at
// the end. Key groups jj >= JN lie wholly past the sequence end: left at 0 (masked later).
template <int JN, int NR>
__device__ __forceinline__ void score_tile(const float* Qs, const float* Ks, int rb, int tx,
                                           float (&s)[NR][4]) {
  uint64_t s2[NR][JN];
#pragma unroll
  for (int i = 0; i < NR; ++i)
#pragma unroll
    for (int jj = 0; jj < JN; ++jj) s2[i][jj] = 0ull;
#pragma unroll 2
  for (int c = 0; c < 64; c += 4) {
    ulonglong2 kv[JN], qv[NR];
#pragma unroll
    for (int jj = 0; jj < JN; ++jj) kv[jj] = ld2x2(Ks + (tx + 16 * jj) * LD + c);
#pragma unroll
    for (int i = 0; i < NR; ++i) qv[i] = ld2x2(Qs + (rb + 2 * i) * LD + c);
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int jj = 0; jj < JN; ++jj) s2[i][jj] = fma2(qv[i].x, kv[jj].x, s2[i][jj]);
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int jj = 0; jj < JN; ++jj) s2[i][jj] = fma2(qv[i].y, kv[jj].y, s2[i][jj]);
  }
#pragma unroll
  for (int i = 0; i < NR; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) s[i][jj] = jj < JN ? sum2(s2[i][jj < JN ? jj : 0]) : 0.0f;
}

template <int RPT, bool CAUSAL>
__global__ void __launch_bounds__(FWD_THREADS, 3) fwd_ffma_kernel(const FwdArgs a) {
  constexpr int BM = 8 * RPT;
  extern __shared__ float4 smem4[];
  float* Qs = reinterpret_cast<float*>(smem4);  // [BM][LD]
  float* Ks = Qs + BM * LD;                     // [64][LD]
  float* Vs = Ks + FWD_BN * LD;                 // [64][LD]
  float* Ps = Vs + FWD_BN * LD;                 // [BM][LDP], query-major; warp w its own rows

  griddep_wait();  // q, k, v may come from the previous kernel on the stream
  griddep_launch_dependents();
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int ty = lane >> 4, tx = lane & 15;
  const int BH = a.B * a.H;
  int qt, bh;
  if (CAUSAL) {
    // Longest tiles first (tile t sees t + 1 key tiles): the last wave is the short ones.
    qt = a.n_qtiles - 1 - static_cast<int>(blockIdx.x / BH);
    bh = static_cast<int>(blockIdx.x % BH);
  } else {
    // The query tiles of one (batch, head) run side by side and share K, V through L2.
    qt = static_cast<int>(blockIdx.x % a.n_qtiles);
    bh = static_cast<int>(blockIdx.x / a.n_qtiles);
  }
  const int b = bh / a.H, h = bh % a.H;
  const int q0 = qt * BM;
  const int S = a.S;
  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* kp = a.k + b * a.k_sb + h * a.k_sh;
  const float* vp = a.v + b * a.v_sb + h * a.v_sh;

  const int k_end = CAUSAL ? min(S, q0 + BM) : S;

  load_tile_async<BM, FWD_THREADS>(Qs, qp, a.q_ss, q0, S);
  load_tile_async<FWD_BN, FWD_THREADS>(Ks, kp, a.k_ss, 0, S);
  cp_async_commit();

  const int rb = 2 * RPT * w + ty;  // this thread's rows: rb + 2i, i < RPT
  // x = (q.k) * scale (exact for a power-of-two scale, as in the composed path), p = e^(x - m)
  // with CUDA's expf. lpart is this thread's share
  // of the row sum (its 4 keys per tile, rescaled like O); the 16 shares of a row are added once,
  // after the last tile.
  // acc2[i][0] holds dims 4tx, 4tx + 1 of row rb + 2i, acc2[i][1] dims 4tx + 2, 4tx + 3.
  float m[RPT], lpart[RPT];
  uint64_t acc2[RPT][2];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    m[i] = -INFINITY;
    lpart[i] = 0.0f;
    acc2[i][0] = acc2[i][1] = 0ull;
  }

  for (int k0 = 0; k0 < k_end; k0 += FWD_BN) {
    // K(k0) (and the first time Q) has landed for every thread, and every thread is done with
    // the previous tile's V and P: V(k0) may overwrite Vs.
    cp_async_wait_all();
    __syncthreads();
    load_tile_async<FWD_BN, FWD_THREADS>(Vs, vp, a.v_ss, k0, S);
    cp_async_commit();

    // Dead work is skipped, uniformly per tile: the key groups wholly past the sequence end of
    // a 33..48-key last tile. The skipped terms are masked scores and products with P = 0: the
    // live results are the same bits either way. (Two instantiations only, for code size and
    // registers; shorter last tiles compute their dead groups and mask them. Skipping whole dead
    // warps measured slower: the branch costs registers.)
    const int jn = min(4, (S - k0 + 15) / 16);
    float s[RPT][4];
    if (jn == 3)
      score_tile<3, RPT>(Qs, Ks, rb, tx, s);
    else
      score_tile<4, RPT>(Qs, Ks, rb, tx, s);

    // Masks only where the tile crosses the sequence end or the causal diagonal (block-uniform).
    const bool edge = (k0 + FWD_BN > S) || (CAUSAL && k0 + FWD_BN - 1 > q0);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      float x[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) x[jj] = s[i][jj] * a.scale;
      if (edge) {
        const int qi = q0 + rb + 2 * i;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = k0 + tx + 16 * jj;
          if (!(j < S && !(CAUSAL && j > qi))) x[jj] = -INFINITY;
        }
      }
      float tmax = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
      tmax = half_warp_max(tmax);
      const float m_new = fmaxf(m[i], tmax);
      // Every row has a live key in its first tile, so m_new is finite; the guard keeps a fully
      // masked row at p = 0 instead of NaN all the same.
      const float mu = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = expf(m[i] - mu);
      float psum = 0.0f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float pr = expf(x[jj] - mu);
        Ps[(rb + 2 * i) * LDP + tx + 16 * jj] = pr;
        psum += pr;
      }
      lpart[i] = fmaf(lpart[i], alpha, psum);
      m[i] = m_new;
      const uint64_t al = dup2(alpha);
      acc2[i][0] = mul2(acc2[i][0], al);
      acc2[i][1] = mul2(acc2[i][1], al);
    }
    // V(k0) has landed, every P is written, and every thread is done with Ks: K(k0 + 64) may
    // overwrite Ks while P V runs.
    cp_async_wait_all();
    __syncthreads();
    if (k0 + FWD_BN < k_end) {
      load_tile_async<FWD_BN, FWD_THREADS>(Ks, kp, a.k_ss, k0 + FWD_BN, S);
      cp_async_commit();
    }

    // O += P V, keys j = k0 .. in order for every element (key groups past the end hold P = 0).
    // Packed FMAs, accumulators paired along dims ((e, e + 1) of the float4 read from V), the P
    // element broadcast: the same fmaf per element as scalar code.
    const int jlim = jn == 3 ? 48 : 64;
#pragma unroll 8  // (unroll 2 / 4 / 8: 167.6 / 164.4 / 162.6 us at the canvas shape)
    for (int j = 0; j < jlim; j += 4) {
      ulonglong2 vv[4];
      float4 pv[RPT];
#pragma unroll
      for (int t = 0; t < 4; ++t) vv[t] = ld2x2(Vs + (j + t) * LD + 4 * tx);
#pragma unroll
      for (int i = 0; i < RPT; ++i) pv[i] = ld4(Ps + (rb + 2 * i) * LDP + j);
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const uint64_t pr = dup2(f4c(pv[i], t));
          acc2[i][0] = fma2(pr, vv[t].x, acc2[i][0]);
          acc2[i][1] = fma2(pr, vv[t].y, acc2[i][1]);
        }
    }
  }

#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    // DETERMINISM: the row sum is the butterfly of the 16 per-thread shares, in a fixed order.
    const float l = half_warp_sum(lpart[i]);
    const int qi = q0 + rb + 2 * i;
    if (qi >= S) continue;
    float4* dst = reinterpret_cast<float4*>(
        a.o + ((static_cast<int64_t>(b) * S + qi) * a.H + h) * 64 + 4 * tx);
    // O = acc / l with one rounding (IEEE division), once per output element.
    const float2 lo = split2(acc2[i][0]), hi = split2(acc2[i][1]);
    *dst = make_float4(__fdiv_rn(lo.x, l), __fdiv_rn(lo.y, l), __fdiv_rn(hi.x, l),
                       __fdiv_rn(hi.y, l));
    if (tx == 0) a.lse[static_cast<int64_t>(bh) * S + qi] = m[i] + logf(l);
  }
}

}  // namespace

int fwd_tile_rows(int64_t seq) {
  const int64_t pad64 = (64 - seq % 64) % 64, pad48 = (48 - seq % 48) % 48;
  return pad48 < pad64 ? 48 : 64;
}

cudaError_t setup_fwd_attributes() {
  cudaError_t e = cudaSuccess;
  auto set = [&](const void* fn, int floats) {
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(floats * sizeof(float)));
  };
  set(reinterpret_cast<const void*>(fwd_ffma_kernel<8, false>), fwd_smem_floats<8>());
  set(reinterpret_cast<const void*>(fwd_ffma_kernel<8, true>), fwd_smem_floats<8>());
  set(reinterpret_cast<const void*>(fwd_ffma_kernel<6, false>), fwd_smem_floats<6>());
  set(reinterpret_cast<const void*>(fwd_ffma_kernel<6, true>), fwd_smem_floats<6>());
  return e;
}

cudaError_t launch_fwd(const FwdArgs& args, int causal, cudaStream_t stream) {
  FwdArgs a = args;
  const int bm = fwd_tile_rows(a.S);
  a.n_qtiles = (a.S + bm - 1) / bm;
  const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(a.n_qtiles) * a.B * a.H));
  const dim3 block(FWD_THREADS);
  if (bm == 48) {
    const size_t smem = fwd_smem_floats<6>() * sizeof(float);
    return causal ? launch_pdl(fwd_ffma_kernel<6, true>, grid, block, smem, stream, a)
                  : launch_pdl(fwd_ffma_kernel<6, false>, grid, block, smem, stream, a);
  }
  const size_t smem = fwd_smem_floats<8>() * sizeof(float);
  return causal ? launch_pdl(fwd_ffma_kernel<8, true>, grid, block, smem, stream, a)
                : launch_pdl(fwd_ffma_kernel<8, false>, grid, block, smem, stream, a);
}

}  // namespace cfa
