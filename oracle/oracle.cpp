// SPDX-License-Identifier: MIT OR Apache-2.0
//
// TEST INFRASTRUCTURE -- the CPU oracle. Only tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline legs may load or run this file's library; the product path never does.
//
// A restatement, in C++, of candle-fused-attn's CPU composed path, the reference's own oracle:
//   gather_cpu         src/lib.rs:223-238   strided [b, h, s, d] operand -> contiguous
//   composed_forward   src/lib.rs:241-259   scores = (q k^T) * scale (+ causal bias), softmax by
//                                           max / exp / sum / div, o = p v, L = max + log(sum)
//   causal_bias        src/lib.rs:262-267   -inf where j > i
//   composed_backward  src/lib.rs:271-299   p = exp(q k^T * scale - L) (* keep mask), dv = p^T dO,
//                                           dp = dO v^T, D = rowsum(dO o O), ds = p o (dp - D),
//                                           dq = (ds k) * scale, dk = (ds^T q) * scale
//   cpu_output         src/lib.rs:318-323   O written [b, s, h, d]
//   qkv bwd concat     src/lib.rs:581-588   dq, dk, dv interleaved as [b, s, 3, h, d]
//   matmul             examples/tutorial.rs:110, :113   the training step's projection
//                                           x.broadcast_matmul(w_qkv) and its weight gradient
// in fp32 (the parity target and the timed CPU baseline) and fp64 (the accuracy reference of
// bench/compare.py:506-536). Same operation order as the composed graph: each matmul sums over its
// inner index in increasing order; the scale multiplies the finished product.
//
// Parity pinning: the reference's CPU path runs on candle-core 0.11.0 / gemm 0.18.2-0.19.0, which
// cannot be built in this image (no cargo), so its bit-level summation order is not reproducible.
// This restatement is pinned by tolerance against outputs of the reference's own CUDA kernel
// (kernels/fused_attn.cu, built from source for sm_100a) stored in tests/golden/, at the band the
// reference's tests use between its CUDA and CPU paths (tests/parity.rs:210-221, 5e-6 max-abs).
//
// Memory: the composed path materialises [s, s] scores per (b, h); this restatement processes one
// (b, h) slice at a time and its rows in blocks of ROW_BLOCK, which changes no per-row arithmetic
// and keeps s = 8192 within a few MB per thread. Slices run in parallel on `threads` std::threads
// (0 = every hardware thread); each slice's arithmetic is independent of the thread count.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <algorithm>
#include <atomic>
#include <thread>

namespace {

constexpr int64_t ROW_BLOCK = 64;

// fn(bh) for bh in [begin, end), on `threads` threads pulling slices from a shared counter.
template <typename Fn>
void parallel_slices(int64_t begin, int64_t end, int threads, Fn fn) {
  if (threads < 1) threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  threads = static_cast<int>(std::min<int64_t>(threads, std::max<int64_t>(1, end - begin)));
  std::atomic<int64_t> next(begin);
  auto worker = [&] {
    for (int64_t bh = next.fetch_add(1); bh < end; bh = next.fetch_add(1)) fn(bh);
  };
  if (threads == 1) {
    worker();
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(static_cast<size_t>(threads));
  for (int t = 0; t < threads; ++t) pool.emplace_back(worker);
  for (auto& th : pool) th.join();
}

// gather_cpu (src/lib.rs:223-238): [s][d] of batch b, head h through (sb, sh, ss) strides.
template <typename T, typename Src>
void gather(const Src* base, const int64_t st[3], int64_t b, int64_t h, int64_t S, int64_t D,
            T* out) {
  const Src* p = base + b * st[0] + h * st[1];
  for (int64_t i = 0; i < S; ++i)
    for (int64_t c = 0; c < D; ++c) out[i * D + c] = static_cast<T>(p[i * st[2] + c]);
}

template <typename T>
T texp(T x) {
  return std::exp(x);
}
template <typename T>
T tlog(T x) {
  return std::log(x);
}

// One (b, h) slice of composed_forward. q, k, v: [S][D]. o: [S][D], l: [S].
template <typename T>
void forward_slice(const T* q, const T* k, const T* v, int64_t S, int64_t D, T scale, bool causal,
                   T* o, T* l) {
  std::vector<T> kt(static_cast<size_t>(D * S));  // k^T: [D][S]
  for (int64_t j = 0; j < S; ++j)
    for (int64_t c = 0; c < D; ++c) kt[c * S + j] = k[j * D + c];
  std::vector<T> sc(static_cast<size_t>(ROW_BLOCK * S));
  for (int64_t r0 = 0; r0 < S; r0 += ROW_BLOCK) {
    const int64_t rn = std::min(ROW_BLOCK, S - r0);
    for (int64_t r = 0; r < rn; ++r) {
      const int64_t i = r0 + r;
      T* srow = sc.data() + r * S;
      // scores = q k^T, summed over c in order; then * scale (src/lib.rs:248)
      for (int64_t j = 0; j < S; ++j) srow[j] = T(0);
      for (int64_t c = 0; c < D; ++c) {
        const T qc = q[i * D + c];
        const T* kr = kt.data() + c * S;
        for (int64_t j = 0; j < S; ++j) srow[j] += qc * kr[j];
      }
      for (int64_t j = 0; j < S; ++j) srow[j] = srow[j] * scale;
      if (causal)  // + causal_bias (src/lib.rs:249-253)
        for (int64_t j = i + 1; j < S; ++j) srow[j] = -INFINITY;
      // max / exp / sum / div (src/lib.rs:254-256)
      T mx = -INFINITY;
      for (int64_t j = 0; j < S; ++j) mx = std::max(mx, srow[j]);
      T sum = T(0);
      for (int64_t j = 0; j < S; ++j) {
        srow[j] = texp(srow[j] - mx);
        sum += srow[j];
      }
      for (int64_t j = 0; j < S; ++j) srow[j] = srow[j] / sum;
      // o = p v, summed over j in order (src/lib.rs:257)
      T* orow = o + i * D;
      for (int64_t c = 0; c < D; ++c) orow[c] = T(0);
      for (int64_t j = 0; j < S; ++j) {
        const T pj = srow[j];
        const T* vr = v + j * D;
        for (int64_t c = 0; c < D; ++c) orow[c] += pj * vr[c];
      }
      l[i] = mx + tlog(sum);  // L = max + log(sum) (src/lib.rs:258)
    }
  }
}

// One (b, h) slice of composed_backward. Outputs dq, dk, dv: [S][D].
template <typename T>
void backward_slice(const T* q, const T* k, const T* v, const T* o, const T* l, const T* dout,
                    int64_t S, int64_t D, T scale, bool causal, T* dq, T* dk, T* dv) {
  std::vector<T> kt(static_cast<size_t>(D * S)), vt(static_cast<size_t>(D * S));
  for (int64_t j = 0; j < S; ++j)
    for (int64_t c = 0; c < D; ++c) {
      kt[c * S + j] = k[j * D + c];
      vt[c * S + j] = v[j * D + c];
    }
  std::fill(dk, dk + S * D, T(0));
  std::fill(dv, dv + S * D, T(0));
  std::vector<T> p(static_cast<size_t>(S)), ds(static_cast<size_t>(S));
  for (int64_t i = 0; i < S; ++i) {
    // p = exp(q k^T * scale - L) (src/lib.rs:286-292), keep mask (src/lib.rs:290-293)
    for (int64_t j = 0; j < S; ++j) p[j] = T(0);
    for (int64_t c = 0; c < D; ++c) {
      const T qc = q[i * D + c];
      const T* kr = kt.data() + c * S;
      for (int64_t j = 0; j < S; ++j) p[j] += qc * kr[j];
    }
    for (int64_t j = 0; j < S; ++j) p[j] = texp(p[j] * scale - l[i]);
    if (causal)
      for (int64_t j = i + 1; j < S; ++j) p[j] = T(0);
    // dv += p^T dO: row i's term, rows in increasing order (src/lib.rs:294)
    for (int64_t j = 0; j < S; ++j) {
      const T pj = p[j];
      T* dvr = dv + j * D;
      for (int64_t c = 0; c < D; ++c) dvr[c] += pj * dout[i * D + c];
    }
    // dp = dO v^T (src/lib.rs:295)
    for (int64_t j = 0; j < S; ++j) ds[j] = T(0);
    for (int64_t c = 0; c < D; ++c) {
      const T gc = dout[i * D + c];
      const T* vr = vt.data() + c * S;
      for (int64_t j = 0; j < S; ++j) ds[j] += gc * vr[j];
    }
    // D = rowsum(dO o O) (src/lib.rs:296)
    T dsum = T(0);
    for (int64_t c = 0; c < D; ++c) dsum += dout[i * D + c] * o[i * D + c];
    // ds = p o (dp - D) (src/lib.rs:297)
    for (int64_t j = 0; j < S; ++j) ds[j] = p[j] * (ds[j] - dsum);
    // dq = (ds k) * scale (src/lib.rs:298)
    for (int64_t c = 0; c < D; ++c) dq[i * D + c] = T(0);
    for (int64_t j = 0; j < S; ++j) {
      const T dj = ds[j];
      const T* kr = k + j * D;
      for (int64_t c = 0; c < D; ++c) dq[i * D + c] += dj * kr[c];
    }
    for (int64_t c = 0; c < D; ++c) dq[i * D + c] = dq[i * D + c] * scale;
    // dk += ds^T q: row i's term (src/lib.rs:299)
    for (int64_t j = 0; j < S; ++j) {
      const T dj = ds[j];
      T* dkr = dk + j * D;
      for (int64_t c = 0; c < D; ++c) dkr[c] += dj * q[i * D + c];
    }
  }
  for (int64_t e = 0; e < S * D; ++e) dk[e] = dk[e] * scale;
}

template <typename T>
void run_forward(const float* q, const int64_t qs[3], const float* k, const int64_t ks[3],
                 const float* v, const int64_t vs[3], int64_t B, int64_t H, int64_t S, int64_t D,
                 double scale, int causal, T* o, T* lse, int threads, int64_t bh_begin,
                 int64_t bh_end) {
  (void)B;
  parallel_slices(bh_begin, bh_end, threads, [&](int64_t bh) {
    const int64_t b = bh / H, h = bh % H;
    std::vector<T> tq(static_cast<size_t>(S * D)), tk(tq.size()), tv(tq.size()), to(tq.size()),
        tl(static_cast<size_t>(S));
    gather(q, qs, b, h, S, D, tq.data());
    gather(k, ks, b, h, S, D, tk.data());
    gather(v, vs, b, h, S, D, tv.data());
    forward_slice<T>(tq.data(), tk.data(), tv.data(), S, D, static_cast<T>(scale), causal != 0,
                     to.data(), tl.data());
    for (int64_t i = 0; i < S; ++i) {
      std::memcpy(o + ((b * S + i) * H + h) * D, to.data() + i * D, sizeof(T) * D);
      lse[bh * S + i] = tl[i];
    }
  });
}

template <typename T>
void run_backward(const float* q, const int64_t qs[3], const float* k, const int64_t ks[3],
                  const float* v, const int64_t vs[3], const T* o, const T* lse, const float* dout,
                  const int64_t dos[3], int64_t B, int64_t H, int64_t S, int64_t D, double scale,
                  int causal, T* dqkv, int threads, int64_t bh_begin, int64_t bh_end) {
  (void)B;
  parallel_slices(bh_begin, bh_end, threads, [&](int64_t bh) {
    const int64_t b = bh / H, h = bh % H;
    const size_t n = static_cast<size_t>(S * D);
    std::vector<T> tq(n), tk(n), tv(n), tg(n), to(n), tl(static_cast<size_t>(S)), dq(n), dk(n),
        dv(n);
    gather(q, qs, b, h, S, D, tq.data());
    gather(k, ks, b, h, S, D, tk.data());
    gather(v, vs, b, h, S, D, tv.data());
    gather(dout, dos, b, h, S, D, tg.data());
    for (int64_t i = 0; i < S; ++i) {  // O is [b, s, h, d] dense
      std::memcpy(to.data() + i * D, o + ((b * S + i) * H + h) * D, sizeof(T) * D);
      tl[i] = lse[bh * S + i];
    }
    backward_slice<T>(tq.data(), tk.data(), tv.data(), to.data(), tl.data(), tg.data(), S, D,
                      static_cast<T>(scale), causal != 0, dq.data(), dk.data(), dv.data());
    for (int64_t i = 0; i < S; ++i) {
      T* row = dqkv + (b * S + i) * 3 * H * D + h * D;
      std::memcpy(row, dq.data() + i * D, sizeof(T) * D);
      std::memcpy(row + H * D, dk.data() + i * D, sizeof(T) * D);
      std::memcpy(row + 2 * H * D, dv.data() + i * D, sizeof(T) * D);
    }
  });
}

// C = A B, the contraction of candle's broadcast_matmul in the reference's training step
// (examples/tutorial.rs:110; the step's weight gradient x^T dqkv is the same product on transposed
// operands). candle-core 0.11.0 computes it on the CPU with the gemm crate (0.18.2 / 0.19.0 in
// Cargo.lock): FMA micro-kernels whose blocking order cannot be reproduced without that crate, so
// this restates the product itself -- every C(i, j) sums its k products in increasing k order, one
// fused multiply-add per product, in T. Rows of C run in parallel; the order within a row does not
// depend on the thread count. A(i, p) = a[i a_rs + p a_cs], B(p, j) = b[p b_rs + j b_cs], C dense.
template <typename T>
void run_matmul(const float* a, int64_t a_rs, int64_t a_cs, const float* b, int64_t b_rs,
                int64_t b_cs, T* c, int64_t m, int64_t n, int64_t k, int threads) {
  parallel_slices(0, m, threads, [&](int64_t i) {
    T* row = c + i * n;
    std::vector<T> brow(static_cast<size_t>(n));
    for (int64_t j = 0; j < n; ++j) row[j] = T(0);
    for (int64_t p = 0; p < k; ++p) {
      const T x = static_cast<T>(a[i * a_rs + p * a_cs]);
      for (int64_t j = 0; j < n; ++j) brow[j] = static_cast<T>(b[p * b_rs + j * b_cs]);
      for (int64_t j = 0; j < n; ++j) row[j] = std::fma(x, brow[j], row[j]);
    }
  });
}

}  // namespace

extern "C" {

// Forward over (b, h) slices [bh_begin, bh_end) (all: 0, B*H). Inputs are fp32 (the op's dtype)
// through (batch, head, seq) strides; outputs O [b, s, h, d] and L [b, h, s], fp32 or fp64.
void oracle_fwd_f32(const float* q, const int64_t* qs, const float* k, const int64_t* ks,
                    const float* v, const int64_t* vs, int64_t B, int64_t H, int64_t S, int64_t D,
                    double scale, int causal, float* o, float* lse, int threads, int64_t bh_begin,
                    int64_t bh_end) {
  run_forward<float>(q, qs, k, ks, v, vs, B, H, S, D, scale, causal, o, lse, threads, bh_begin,
                     bh_end);
}

void oracle_fwd_f64(const float* q, const int64_t* qs, const float* k, const int64_t* ks,
                    const float* v, const int64_t* vs, int64_t B, int64_t H, int64_t S, int64_t D,
                    double scale, int causal, double* o, double* lse, int threads,
                    int64_t bh_begin, int64_t bh_end) {
  run_forward<double>(q, qs, k, ks, v, vs, B, H, S, D, scale, causal, o, lse, threads, bh_begin,
                      bh_end);
}

// Backward over (b, h) slices [bh_begin, bh_end): dqkv [b, s, 3, h, d] from the forward's O, L
// (same precision as the output) and dO (fp32, strided).
void oracle_bwd_f32(const float* q, const int64_t* qs, const float* k, const int64_t* ks,
                    const float* v, const int64_t* vs, const float* o, const float* lse,
                    const float* dout, const int64_t* dos, int64_t B, int64_t H, int64_t S,
                    int64_t D, double scale, int causal, float* dqkv, int threads,
                    int64_t bh_begin, int64_t bh_end) {
  run_backward<float>(q, qs, k, ks, v, vs, o, lse, dout, dos, B, H, S, D, scale, causal, dqkv,
                      threads, bh_begin, bh_end);
}

void oracle_bwd_f64(const float* q, const int64_t* qs, const float* k, const int64_t* ks,
                    const float* v, const int64_t* vs, const double* o, const double* lse,
                    const float* dout, const int64_t* dos, int64_t B, int64_t H, int64_t S,
                    int64_t D, double scale, int causal, double* dqkv, int threads,
                    int64_t bh_begin, int64_t bh_end) {
  run_backward<double>(q, qs, k, ks, v, vs, o, lse, dout, dos, B, H, S, D, scale, causal, dqkv,
                       threads, bh_begin, bh_end);
}

// C [m, n] dense = A B over fp32 inputs through (row, column) strides, in fp32 or fp64.
void oracle_matmul_f32(const float* a, int64_t a_rs, int64_t a_cs, const float* b, int64_t b_rs,
                       int64_t b_cs, float* c, int64_t m, int64_t n, int64_t k, int threads) {
  run_matmul<float>(a, a_rs, a_cs, b, b_rs, b_cs, c, m, n, k, threads);
}

void oracle_matmul_f64(const float* a, int64_t a_rs, int64_t a_cs, const float* b, int64_t b_rs,
                       int64_t b_cs, double* c, int64_t m, int64_t n, int64_t k, int threads) {
  run_matmul<double>(a, a_rs, a_cs, b, b_rs, b_cs, c, m, n, k, threads);
}

int oracle_max_threads(void) {
  return static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
}

}  // extern "C"
