// SPDX-License-Identifier: MIT OR Apache-2.0
//
// Head dims 32 and 128: the forward, the D prep and the one-pass backward of csrc/fwd_ffma.cu and
// csrc/bwd_ffma.cu, templated on the head dim D. The reference's CUDA path takes head_dim 64 only
// (src/lib.rs:91 CUDA_HEAD_DIM, src/cuda.rs:85-93) and lists 32 and 128 as later work
// (ROADMAP.md, "head_dim 32 and 128"); its CPU path takes any head dim, and that path is the
// oracle these kernels are checked against (tests/test_head_dims_gpu.py).
//
// The head-dim-64 kernels stay as they are; these follow the same design, with the tiles resized
// so that registers and shared memory fit:
//   forward   D = 32:  64 or 48 queries per block, each thread 8 or 6 rows x 4 keys (S) and x 2
//                      dims (O)
//             D = 128: 48 queries per block, each thread 6 rows x 4 keys (S) and x 8 dims (O),
//                      the 8 dims as two float4 64 apart (conflict-free loads); 2 blocks per SM.
//             (D = 32: the tile height that pads the fewer query rows at the sequence length.)
//   backward  D = 32:  256 threads per 64-key block, as head dim 64 with 2 dims per thread
//             D = 128: 512 threads per 64-key block (one block per SM, 176 KB of shared memory):
//                      phase 1 4 rows x 4 keys per thread, phase 2 4 keys x 8 dims (dV, dK),
//                      phase 3 4 rows x 4 dims, the two 64-dim halves on the two warp groups.
// Every sum keeps the fixed orders of the head-dim-64 kernels: scores as an even-d plus an odd-d
// chain, the softmax butterflies, O and dK/dV over keys / queries in index order, D in fp64, dQ
// over key blocks in key-block order (turn chain or no-wait partials, the same bits). Results are
// bit-identical across reruns, batch splits and workspace sizes.
#include "cfa_common.cuh"

namespace cfa {
namespace {

template <int D>
struct Hd;
// The forward's rows per thread: two candidates per head dim (query tiles of 8 RPT rows), the one
// that pads fewer rows at the sequence length taken (hd_fwd_rows; rows are independent, so the
// choice changes no bit), and blocks per SM.
template <>
struct Hd<32> {
  static constexpr int RPT_A = 8, RPT_B = 6;  // 64- or 48-query tiles
  static constexpr int FWD_MINB = 3;          // forward blocks per SM (registers)
};
template <>
struct Hd<128> {
  // 48-query tiles at every length: against 32-query tiles (4 rows per thread) they measured
  // faster at every shape tried (canvas-shaped 185 -> 158 us, s = 4096 causal 917 -> 820 us).
  static constexpr int RPT_A = 6, RPT_B = 6;
  static constexpr int FWD_MINB = 2;          // (shared memory: 107.3 KB per block)
};

template <int RPT>
__host__ __device__ constexpr int fwd_bm() {
  return 8 * RPT;  // 4 warps x 2 half-warps x RPT rows
}

// Row stride of the [rows][D] tiles: D + 4 floats, rows 16-byte aligned and 4 banks apart.
template <int D>
__host__ __device__ constexpr int ldh() {
  return D + 4;
}

template <int D, int RPT>
__host__ __device__ constexpr int hd_fwd_smem_floats() {
  return (fwd_bm<RPT>() + 2 * 64) * ldh<D>() + fwd_bm<RPT>() * LDP;
}

template <int D>
__host__ __device__ constexpr int hd_bwd_smem_floats() {
  return 4 * 64 * ldh<D>() + 2 * 64 * LDP + 2 * 64 + 4;
}

// ROWS rows of a strided [seq, D] slice starting at row0 into a [ROWS][D + 4] tile (zero past seq;
// the address given for such rows is row0's, which is < seq).
template <int ROWS, int NT, int D>
__device__ __forceinline__ void load_rows_async(float* dst, const float* __restrict__ src,
                                                int64_t s_stride, int row0, int seq) {
  constexpr int C = D / 4;
#pragma unroll
  for (int idx = threadIdx.x; idx < ROWS * C; idx += NT) {
    const int r = idx / C, c4 = idx % C;
    const int row = row0 + r;
    const bool ok = row < seq;
    const float* g = src + static_cast<int64_t>(ok ? row : row0) * s_stride + 4 * c4;
    cp_async16(dst + r * ldh<D>() + 4 * c4, g, ok ? 16 : 0);
  }
}

// S = A B^T for NR rows (rb + 2i) and the first JN of 4 key groups (keys tx + 16jj): an even-d
// chain plus an odd-d chain per score, as the head-dim-64 kernels do. Groups >= JN are left at 0.
template <int JN, int NR, int D>
__device__ __forceinline__ void scores(const float* As, const float* Bs, int rb, int tx,
                                       float (&s)[NR][4]) {
  uint64_t s2[NR][JN];
#pragma unroll
  for (int i = 0; i < NR; ++i)
#pragma unroll
    for (int jj = 0; jj < JN; ++jj) s2[i][jj] = 0ull;
#pragma unroll 2
  for (int c = 0; c < D; c += 4) {
    ulonglong2 bv[JN], av[NR];
#pragma unroll
    for (int jj = 0; jj < JN; ++jj) bv[jj] = ld2x2(Bs + (tx + 16 * jj) * ldh<D>() + c);
#pragma unroll
    for (int i = 0; i < NR; ++i) av[i] = ld2x2(As + (rb + 2 * i) * ldh<D>() + c);
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int jj = 0; jj < JN; ++jj) s2[i][jj] = fma2(av[i].x, bv[jj].x, s2[i][jj]);
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
      for (int jj = 0; jj < JN; ++jj) s2[i][jj] = fma2(av[i].y, bv[jj].y, s2[i][jj]);
  }
#pragma unroll
  for (int i = 0; i < NR; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) s[i][jj] = jj < JN ? sum2(s2[i][jj < JN ? jj : 0]) : 0.0f;
}

// This thread's D / 16 output dims of a row, as register pairs: D = 32 -> dims 2tx, 2tx + 1 (one
// pair); D = 128 -> dims 4tx .. 4tx + 3 and 64 + 4tx .. 64 + 4tx + 3 (four pairs).
template <int D>
struct Dims;
template <>
struct Dims<32> {
  static constexpr int NP = 1;
  __device__ __forceinline__ static void load(const float* row, int tx, uint64_t (&v)[1]) {
    v[0] = *reinterpret_cast<const uint64_t*>(row + 2 * tx);
  }
  __device__ __forceinline__ static void load_f(const float* row, int tx, float (&v)[2]) {
    const float2 x = *reinterpret_cast<const float2*>(row + 2 * tx);
    v[0] = x.x;
    v[1] = x.y;
  }
};
template <>
struct Dims<128> {
  static constexpr int NP = 4;
  __device__ __forceinline__ static void load(const float* row, int tx, uint64_t (&v)[4]) {
    const ulonglong2 a = ld2x2(row + 4 * tx), b = ld2x2(row + 64 + 4 * tx);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  }
  __device__ __forceinline__ static void load_f(const float* row, int tx, float (&v)[8]) {
    const float4 a = ld4(row + 4 * tx), b = ld4(row + 64 + 4 * tx);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = a.z;
    v[3] = a.w;
    v[4] = b.x;
    v[5] = b.y;
    v[6] = b.z;
    v[7] = b.w;
  }
};

// Store this thread's D / 16 dims of a row (the layout of Dims<D>) into row `dst`.
template <int D>
__device__ __forceinline__ void store_dims(float* dst, int tx, const float (&v)[D / 16]) {
  if constexpr (D == 32) {
    *reinterpret_cast<float2*>(dst + 2 * tx) = make_float2(v[0], v[1]);
  } else {
    *reinterpret_cast<float4*>(dst + 4 * tx) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(dst + 64 + 4 * tx) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// ---------------------------------------------------------------------------------------------
// Forward: csrc/fwd_ffma.cu's kernel with D-sized tiles (see the header comment).
template <int D, int RPT, bool CAUSAL>
__global__ void __launch_bounds__(FWD_THREADS, Hd<D>::FWD_MINB) hd_fwd_kernel(const FwdArgs a) {
  constexpr int BM = fwd_bm<RPT>(), L = ldh<D>(), NP = Dims<D>::NP;
  extern __shared__ float4 smem4[];
  float* Qs = reinterpret_cast<float*>(smem4);  // [BM][L]
  float* Ks = Qs + BM * L;                      // [64][L]
  float* Vs = Ks + 64 * L;                      // [64][L]
  float* Ps = Vs + 64 * L;                      // [BM][LDP]

  griddep_wait();  // q, k, v may come from the previous kernel on the stream
  griddep_launch_dependents();
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int ty = lane >> 4, tx = lane & 15;
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
  const int q0 = qt * BM;
  const int S = a.S;
  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* kp = a.k + b * a.k_sb + h * a.k_sh;
  const float* vp = a.v + b * a.v_sb + h * a.v_sh;
  const int k_end = CAUSAL ? min(S, q0 + BM) : S;

  load_rows_async<BM, FWD_THREADS, D>(Qs, qp, a.q_ss, q0, S);
  load_rows_async<64, FWD_THREADS, D>(Ks, kp, a.k_ss, 0, S);
  cp_async_commit();

  const int rb = 2 * RPT * w + ty;  // rows rb + 2i
  float m[RPT], lpart[RPT];
  uint64_t acc2[RPT][NP];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    m[i] = -INFINITY;
    lpart[i] = 0.0f;
#pragma unroll
    for (int p = 0; p < NP; ++p) acc2[i][p] = 0ull;
  }

  for (int k0 = 0; k0 < k_end; k0 += 64) {
    cp_async_wait_all();
    __syncthreads();
    load_rows_async<64, FWD_THREADS, D>(Vs, vp, a.v_ss, k0, S);
    cp_async_commit();

    const int jn = min(4, (S - k0 + 15) / 16);
    float s[RPT][4];
    if (jn == 3)
      scores<3, RPT, D>(Qs, Ks, rb, tx, s);
    else
      scores<4, RPT, D>(Qs, Ks, rb, tx, s);

    const bool edge = (k0 + 64 > S) || (CAUSAL && k0 + 63 > q0);
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
#pragma unroll
      for (int p = 0; p < NP; ++p) acc2[i][p] = mul2(acc2[i][p], al);
    }
    cp_async_wait_all();
    __syncthreads();
    if (k0 + 64 < k_end) {
      load_rows_async<64, FWD_THREADS, D>(Ks, kp, a.k_ss, k0 + 64, S);
      cp_async_commit();
    }

    // O += P V over the live key groups, keys in order (groups past the end hold P = 0).
    const int jlim = 16 * jn;
#pragma unroll 8
    for (int j = 0; j < jlim; j += 4) {
      uint64_t vv[4][NP];
      float4 pv[RPT];
#pragma unroll
      for (int t = 0; t < 4; ++t) Dims<D>::load(Vs + (j + t) * L, tx, vv[t]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) pv[i] = ld4(Ps + (rb + 2 * i) * LDP + j);
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const uint64_t pr = dup2(f4c(pv[i], t));
#pragma unroll
          for (int p = 0; p < NP; ++p) acc2[i][p] = fma2(pr, vv[t][p], acc2[i][p]);
        }
    }
  }

#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const float l = half_warp_sum(lpart[i]);
    const int qi = q0 + rb + 2 * i;
    if (qi >= S) continue;
    float ov[D / 16];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const float2 v = split2(acc2[i][p]);
      ov[2 * p] = __fdiv_rn(v.x, l);
      ov[2 * p + 1] = __fdiv_rn(v.y, l);
    }
    store_dims<D>(a.o + ((static_cast<int64_t>(b) * S + qi) * a.H + h) * D, tx, ov);
    if (tx == 0) a.lse[static_cast<int64_t>(bh) * S + qi] = m[i] + logf(l);
  }
}

// ---------------------------------------------------------------------------------------------
// D = rowsum(dO o O) in fp64: 16 lanes per row, D / 16 products per lane in d order (the dims of
// Dims<D>), then the butterfly 1, 2, 4, 8; clears the ticket, error flag and counters.
template <int D>
__global__ void __launch_bounds__(PREP_THREADS) hd_prep_kernel(const PrepArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t gtid = static_cast<int64_t>(blockIdx.x) * PREP_THREADS + threadIdx.x;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * PREP_THREADS;
  for (int64_t z = gtid; z < a.n_zero; z += gstride) a.zero[z] = 0;

  const int64_t rows = static_cast<int64_t>(a.B) * a.H * a.S;
  const int64_t row = gtid >> 4;
  const int c = threadIdx.x & 15;
  double x = 0.0;
  if (row < rows) {
    const int i = static_cast<int>(row % a.S);
    const int64_t bhr = row / a.S;
    const int h = static_cast<int>(bhr % a.H), b = static_cast<int>(bhr / a.H);
    float ov[D / 16], gv[D / 16];
    Dims<D>::load_f(a.o + ((static_cast<int64_t>(b) * a.S + i) * a.H + h) * D, c, ov);
    Dims<D>::load_f(a.d_o + b * a.do_sb + h * a.do_sh + i * a.do_ss, c, gv);
#pragma unroll
    for (int e = 0; e < D / 16; ++e) x = __fma_rn(static_cast<double>(ov[e]), gv[e], x);
  }
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  if (row < rows && c == 0) a.dsum[row] = static_cast<float>(x);
}

// ---------------------------------------------------------------------------------------------
// Backward main kernel: csrc/bwd_ffma.cu's design (phases 1-3, dQ by turn chain or no-wait
// partials, tickets, bounded waits) with the thread layout of the header comment.
template <int D>
struct Bwd;
template <>
struct Bwd<32> {
  static constexpr int NT = 256, WG = 4;   // threads; warps per group
  static constexpr int R1 = 8;             // phase 1 rows per thread (rows rb1 + 2i)
  static constexpr int K2 = 8;             // phase 2 keys per thread
  static constexpr int NP2 = 1;            // phase 2 dim pairs per key pair (dims 2tx, 2tx + 1)
};
template <>
struct Bwd<128> {
  static constexpr int NT = 512, WG = 8;
  static constexpr int R1 = 4;
  static constexpr int K2 = 4;
  static constexpr int NP2 = 4;            // dims 4tx .. + 3 and 64 + 4tx .. + 3
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(Bwd<D>::NT, 256 / (Bwd<D>::NT / 2)) hd_bwd_kernel(const BwdArgs a) {
  constexpr int NT = Bwd<D>::NT, WG = Bwd<D>::WG, R1 = Bwd<D>::R1, K2 = Bwd<D>::K2;
  constexpr int NP2 = Bwd<D>::NP2, L = ldh<D>();
  constexpr int DPT = 2 * NP2;  // phase 2 dims per thread
  extern __shared__ float4 smem4[];
  float* Ks = reinterpret_cast<float*>(smem4);  // [64][L]
  float* Vs = Ks + 64 * L;
  float* Qs = Vs + 64 * L;
  float* dOs = Qs + 64 * L;
  float* Ps = dOs + 64 * L;   // [64][LDP] query-major
  float* dSs = Ps + 64 * LDP;
  float* Lt = dSs + 64 * LDP;
  float* Dt = Lt + 64;
  int* s_int = reinterpret_cast<int*>(Dt + 64);

  griddep_launch_dependents();
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int ty = lane >> 4, tx = lane & 15;
  const int grp = w / WG, wg = w % WG;  // grp 0: S, P, dV; grp 1: dP, dS, dK
  const int S = a.S;

  // The prep kernel's writes (D, the cleared ticket and counters) are awaited before their first
  // use; the no-wait path takes its block index as ticket and loads its first q, k, v, dO tiles
  // meanwhile (as the head-dim-64 kernel does).
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
  const int BH = a.B * a.H;
  const bool bh_major = !CAUSAL && no_wait;
  const int kb = bh_major ? ticket % a.n_kblocks : ticket / BH;
  const int bh = bh_major ? ticket / a.n_kblocks : ticket % BH;
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kb * 64;

  const float* qp = a.q + b * a.q_sb + h * a.q_sh;
  const float* gp = a.d_o + b * a.do_sb + h * a.do_sh;
  const float* lp = a.lse + static_cast<int64_t>(bh) * S;
  const float* dp = a.dsum + static_cast<int64_t>(bh) * S;
  int* turn = a.turn + static_cast<int64_t>(bh) * a.n_qtiles;
  const int64_t row_stride = 3 * static_cast<int64_t>(a.H) * D;
  float* dq_base = a.dqkv + static_cast<int64_t>(b) * S * row_stride + h * D;

  load_rows_async<64, NT, D>(Ks, a.k + b * a.k_sb + h * a.k_sh, a.k_ss, k0, S);
  load_rows_async<64, NT, D>(Vs, a.v + b * a.v_sb + h * a.v_sh, a.v_ss, k0, S);

  // grp 0: dV, grp 1: dK (unscaled). acc2[rp][e]: keys kb2 + 2rp, kb2 + 2rp + 1 (a pair), dim e
  // of this thread's phase 2 dims.
  uint64_t acc2[K2 / 2][DPT];
#pragma unroll
  for (int i = 0; i < K2 / 2; ++i)
#pragma unroll
    for (int e = 0; e < DPT; ++e) acc2[i][e] = 0ull;

  const int rb1 = 2 * R1 * wg + ty;          // phase 1 rows: rb1 + 2i (warp: 2 R1 rows)
  const int kb2 = K2 * (2 * wg + ty);        // phase 2 keys: kb2 .. kb2 + K2 - 1
  // phase 3: rows rb3 + 2r (r < 4), dims d3 .. d3 + 3 (D = 128: the two groups take the halves)
  const int rb3 = D == 32 ? 8 * w + ty : 8 * wg + ty;
  const int d3 = D == 32 ? 2 * tx : 64 * grp + 4 * tx;

  auto load_q_do = [&](int q0) {
    load_rows_async<64, NT, D>(Qs, qp, a.q_ss, q0, S);
    load_rows_async<64, NT, D>(dOs, gp, a.do_ss, q0, S);
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

  const int t_begin = CAUSAL ? k0 / 64 : 0;
  load_q_do(t_begin * 64);
  if (no_wait) griddep_wait();
  load_l_d(t_begin * 64);
  cp_async_commit();
  for (int t = t_begin; t < a.n_qtiles; ++t) {
    const int q0 = t * 64;
    cp_async_wait_all();
    __syncthreads();

    const int jn = min(4, (S - k0 + 15) / 16);
    const int iq = min(64, (S - q0 + 15) / 16 * 16);

    // Phase 1. grp 0: s = Q K^T; grp 1: s = dO V^T (dP).
    {
      const float* As = grp ? dOs : Qs;
      const float* Bs = grp ? Vs : Ks;
      float s[R1][4];
      if (q0 + 2 * R1 * wg >= S) {
#pragma unroll
        for (int i = 0; i < R1; ++i)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) s[i][jj] = 0.0f;
      } else if (jn == 4) {
        scores<4, R1, D>(As, Bs, rb1, tx, s);
      } else if (jn == 3) {
        scores<3, R1, D>(As, Bs, rb1, tx, s);
      } else if (jn == 2) {
        scores<2, R1, D>(As, Bs, rb1, tx, s);
      } else {
        scores<1, R1, D>(As, Bs, rb1, tx, s);
      }
      if (grp == 0) {
        const bool edge = (q0 + 64 > S) || (k0 + 64 > S) || (CAUSAL && k0 + 63 > q0);
#pragma unroll
        for (int i = 0; i < R1; ++i) {
          const int il = rb1 + 2 * i, qi = q0 + il;
          const float li = Lt[il];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int jl = tx + 16 * jj, j = k0 + jl;
            float pr = expf(fmaf(s[i][jj], a.scale, -li));
            if (edge && !(qi < S && j < S && !(CAUSAL && j > qi))) pr = 0.0f;
            Ps[il * LDP + jl] = pr;
          }
        }
      }
      __syncthreads();
      if (grp == 1) {
#pragma unroll
        for (int i = 0; i < R1; ++i) {
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

    // Phase 2. grp 0: dV[j] += sum_i P[i][j] dO[i]; grp 1: dK[j] += sum_i dS[i][j] Q[i]. Pairs
    // along keys, the dO / Q element broadcast; queries in index order.
    {
      const float* Xs = grp ? dSs : Ps;
      const float* Ys = grp ? Qs : dOs;
      const int iw = k0 + kb2 - K2 * ty >= S ? 0 : iq;  // all this warp's keys past the end
#pragma unroll 8
      for (int i = 0; i < iw; ++i) {
        uint64_t xp[K2 / 2];
        if constexpr (K2 == 8) {
          const ulonglong2 xa = ld2x2(Xs + i * LDP + kb2), xb = ld2x2(Xs + i * LDP + kb2 + 4);
          xp[0] = xa.x;
          xp[1] = xa.y;
          xp[2] = xb.x;
          xp[3] = xb.y;
        } else {
          const ulonglong2 xa = ld2x2(Xs + i * LDP + kb2);
          xp[0] = xa.x;
          xp[1] = xa.y;
        }
        float y[DPT];
        Dims<D>::load_f(Ys + i * L, tx, y);
#pragma unroll
        for (int e = 0; e < DPT; ++e) {
          const uint64_t yb = dup2(y[e]);
#pragma unroll
          for (int rp = 0; rp < K2 / 2; ++rp) acc2[rp][e] = fma2(xp[rp], yb, acc2[rp][e]);
        }
      }
    }
    __syncthreads();
    if (t + 1 < a.n_qtiles) {
      load_query_tile(q0 + 64);
      cp_async_commit();
    }

    // Phase 3: the dQ partial pq[r][e] = sum_j dS[rb3 + 2r][j] K[j][d3 + e], keys in order.
    constexpr int E3 = D == 32 ? 2 : 4;
    uint64_t pq2[4][E3 / 2];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int p = 0; p < E3 / 2; ++p) pq2[r][p] = 0ull;
    const int jlim = q0 + (rb3 - ty) >= S ? 0 : 16 * jn;
#pragma unroll 2
    for (int j = 0; j < jlim; j += 4) {
      uint64_t k2[4][E3 / 2];
      float4 d4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if constexpr (E3 == 2) {
          k2[u][0] = *reinterpret_cast<const uint64_t*>(Ks + (j + u) * L + d3);
        } else {
          const ulonglong2 kv = ld2x2(Ks + (j + u) * L + d3);
          k2[u][0] = kv.x;
          k2[u][1] = kv.y;
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) d4[r] = ld4(dSs + (rb3 + 2 * r) * LDP + j);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint64_t ds = dup2(f4c(d4[r], u));
#pragma unroll
          for (int p = 0; p < E3 / 2; ++p) pq2[r][p] = fma2(ds, k2[u][p], pq2[r][p]);
        }
    }
    float pq[4][E3];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int p = 0; p < E3 / 2; ++p) {
        const float2 v = split2(pq2[r][p]);
        pq[r][2 * p] = v.x;
        pq[r][2 * p + 1] = v.y;
      }

    if (a.dq_part != nullptr) {
      float* part = a.dq_part + (static_cast<int64_t>(bh) * a.n_kblocks + kb) * S * D;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int qi = q0 + rb3 + 2 * r;
        if (qi >= S) continue;
        float* dst = part + static_cast<int64_t>(qi) * D + d3;
        if constexpr (E3 == 2)
          __stcg(reinterpret_cast<float2*>(dst), make_float2(pq[r][0], pq[r][1]));
        else
          __stcg(reinterpret_cast<float4*>(dst), make_float4(pq[r][0], pq[r][1], pq[r][2], pq[r][3]));
      }
      continue;
    }
    // Turn chain (long sequences): key blocks add into dQ in index order, each on its turn.
    const int last = CAUSAL ? min(a.n_kblocks - 1, min(S - 1, q0 + 63) / 64) : a.n_kblocks - 1;
    bool go = true;
    if (kb > 0) {
      if (tid == 0) {
        s_int[1] = wait_turn_bounded(turn + t, kb, a.err, a.timeout_ns, a.sink) ? 1 : 0;
        __threadfence();  // ORDER: with the barrier, extends thread 0's acquire to the block
      }
      __syncthreads();
      go = s_int[1] != 0;
    }
    if (go) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int qi = q0 + rb3 + 2 * r;
        if (qi >= S) continue;
        float* dst = dq_base + qi * row_stride + d3;
#pragma unroll
        for (int e = 0; e < E3; ++e) {
          float v = pq[r][e];
          if (kb > 0) v = __ldcg(dst + e) + v;  // through L2: L1 is not coherent across SMs
          if (kb == last) v *= a.scale;
          __stcg(dst + e, v);
        }
      }
    }
    if (kb < last) {
      __threadfence();  // ORDER: this block's dQ stores are visible before the turn passes on
      __syncthreads();
      if (tid == 0) st_release_gpu(turn + t, kb + 1);
    }
  }

  if (a.dq_part != nullptr) {
    // ORDER: partials visible GPU-wide before counting in; the last to count sums them all.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_int[1] = atomicAdd(a.turn + bh, 1);
    __syncthreads();
    if (s_int[1] == a.n_kblocks - 1) {
      __threadfence();
      const float* part = a.dq_part + static_cast<int64_t>(bh) * a.n_kblocks * S * D;
      constexpr int C = D / 4;  // float4 per row
      // DETERMINISM: (((p0 + p1) + p2) + ...) * scale over the contributing key blocks in order.
      for (int idx = tid; idx < S * C; idx += NT) {
        const int i = idx / C, c4 = idx % C;
        const int tq = i / 64;
        const int last = CAUSAL ? min(a.n_kblocks - 1, min(S - 1, tq * 64 + 63) / 64)
                                : a.n_kblocks - 1;
        float4 v = __ldcg(reinterpret_cast<const float4*>(part + static_cast<int64_t>(i) * D + 4 * c4));
        for (int j = 1; j <= last; ++j) {
          const float4 p = __ldcg(reinterpret_cast<const float4*>(
              part + (static_cast<int64_t>(j) * S + i) * D + 4 * c4));
          v = make_float4(v.x + p.x, v.y + p.y, v.z + p.z, v.w + p.w);
        }
        *reinterpret_cast<float4*>(dq_base + i * row_stride + 4 * c4) =
            make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
      }
    }
  }

  // grp 0 stores dV into slot 2, grp 1 stores dK * scale into slot 1.
  float* dst0 = a.dqkv + static_cast<int64_t>(b) * S * row_stride + (grp ? 1 : 2) * a.H * D + h * D;
  const float f = grp ? a.scale : 1.0f;
#pragma unroll
  for (int rp = 0; rp < K2 / 2; ++rp) {
    float lo[DPT], hi[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) {
      const float2 v = split2(acc2[rp][e]);
      lo[e] = v.x * f;
      hi[e] = v.y * f;
    }
    const int j = k0 + kb2 + 2 * rp;
    if (j < S) store_dims<D>(dst0 + j * row_stride, tx, lo);
    if (j + 1 < S) store_dims<D>(dst0 + (j + 1) * row_stride, tx, hi);
  }
}

template <int D>
cudaError_t set_attrs() {
  constexpr int A = Hd<D>::RPT_A, Bq = Hd<D>::RPT_B;
  cudaError_t e = cudaSuccess;
  auto set = [&](const void* fn, int floats) {
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, floats * 4);
  };
  set(reinterpret_cast<const void*>(hd_fwd_kernel<D, A, false>), hd_fwd_smem_floats<D, A>());
  set(reinterpret_cast<const void*>(hd_fwd_kernel<D, A, true>), hd_fwd_smem_floats<D, A>());
  if constexpr (Bq != A) {
    set(reinterpret_cast<const void*>(hd_fwd_kernel<D, Bq, false>), hd_fwd_smem_floats<D, Bq>());
    set(reinterpret_cast<const void*>(hd_fwd_kernel<D, Bq, true>), hd_fwd_smem_floats<D, Bq>());
  }
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(hd_bwd_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             hd_bwd_smem_floats<D>() * 4);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(hd_bwd_kernel<D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             hd_bwd_smem_floats<D>() * 4);
  return e;
}

}  // namespace

template <int D>
int rows_for(int64_t seq) {
  const int a = fwd_bm<Hd<D>::RPT_A>(), b = fwd_bm<Hd<D>::RPT_B>();
  const int64_t pa = (a - seq % a) % a, pb = (b - seq % b) % b;
  return pb < pa ? b : a;
}

template <int D>
cudaError_t launch_fwd_d(const FwdArgs& args, int causal, cudaStream_t stream) {
  constexpr int A = Hd<D>::RPT_A, Bq = Hd<D>::RPT_B;
  FwdArgs a = args;
  const int bm = rows_for<D>(a.S);
  a.n_qtiles = (a.S + bm - 1) / bm;
  const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(a.n_qtiles) * a.B * a.H));
  const dim3 block(FWD_THREADS);
  if (bm == fwd_bm<Bq>()) {
    const size_t smem = hd_fwd_smem_floats<D, Bq>() * 4;
    return causal ? launch_pdl(hd_fwd_kernel<D, Bq, true>, grid, block, smem, stream, a)
                  : launch_pdl(hd_fwd_kernel<D, Bq, false>, grid, block, smem, stream, a);
  }
  const size_t smem = hd_fwd_smem_floats<D, A>() * 4;
  return causal ? launch_pdl(hd_fwd_kernel<D, A, true>, grid, block, smem, stream, a)
                : launch_pdl(hd_fwd_kernel<D, A, false>, grid, block, smem, stream, a);
}

int hd_fwd_rows(int head_dim, int64_t seq) {
  return head_dim == 128 ? rows_for<128>(seq) : rows_for<32>(seq);
}

cudaError_t setup_hd_attributes() {
  cudaError_t e = set_attrs<32>();
  return e == cudaSuccess ? set_attrs<128>() : e;
}

cudaError_t launch_hd_fwd(const FwdArgs& a, int head_dim, int causal, cudaStream_t stream) {
  return head_dim == 32 ? launch_fwd_d<32>(a, causal, stream) : launch_fwd_d<128>(a, causal, stream);
}

cudaError_t launch_hd_bwd_prep(const PrepArgs& a, int head_dim, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(a.B) * a.H * a.S;
  int64_t blocks = (rows * 16 + PREP_THREADS - 1) / PREP_THREADS;
  if (blocks < 1) blocks = 1;
  const dim3 grid(static_cast<unsigned>(blocks));
  return head_dim == 32 ? launch_pdl(hd_prep_kernel<32>, grid, dim3(PREP_THREADS), 0, stream, a)
                        : launch_pdl(hd_prep_kernel<128>, grid, dim3(PREP_THREADS), 0, stream, a);
}

cudaError_t launch_hd_bwd(const BwdArgs& a, int head_dim, int causal, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(a.n_kblocks) * a.B * a.H));
  if (head_dim == 32) {
    const size_t smem = hd_bwd_smem_floats<32>() * 4;
    return causal ? launch_pdl(hd_bwd_kernel<32, true>, grid, dim3(Bwd<32>::NT), smem, stream, a)
                  : launch_pdl(hd_bwd_kernel<32, false>, grid, dim3(Bwd<32>::NT), smem, stream, a);
  }
  const size_t smem = hd_bwd_smem_floats<128>() * 4;
  return causal ? launch_pdl(hd_bwd_kernel<128, true>, grid, dim3(Bwd<128>::NT), smem, stream, a)
                : launch_pdl(hd_bwd_kernel<128, false>, grid, dim3(Bwd<128>::NT), smem, stream, a);
}

}  // namespace cfa
