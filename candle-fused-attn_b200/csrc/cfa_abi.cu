// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The C ABI (include/cfa.h): argument checks, the once-per-device kernel attribute set-up, and
// the launches. This is the B200 replacement of the reference's launch layer, src/cuda.rs: the
// same inputs, the same outputs and layouts, the same stream discipline (everything on the
// caller's stream, no synchronisation), with the checks the reference makes in Rust
// (src/cuda.rs:69-93, src/lib.rs:431-435, :533-538) repeated here so a C caller gets them too.
#include <atomic>
#include <mutex>

#include "cfa_internal.h"

namespace {

using cfa::BwdArgs;
using cfa::FwdArgs;
using cfa::PrepArgs;

constexpr int kMaxDevices = 64;

// Per-device once flags: cudaFuncSetAttribute applies to the current device's context.
struct DeviceOnce {
  std::once_flag flag;
  cudaError_t result = cudaSuccess;
};
DeviceOnce g_fwd_once[kMaxDevices];
DeviceOnce g_bwd_once[kMaxDevices];
DeviceOnce g_hd_once[kMaxDevices];  // head dims 32 and 128
DeviceOnce g_fwd_tc_once[kMaxDevices];
DeviceOnce g_bwd_tc_once[kMaxDevices];
// The head-dim-64 kernel pair of a call, chosen by the entry point (no process-wide state): the
// tensor-core pair (the _d64 and head-dim-generic entry points) or the FFMA pair (the _ffma ones).
// A backward recomputes its forward's scores bit for bit only within one pair.
enum class Pair { kTensorCore, kFfma };
// The host-visible error flag of cfa_error_sink, as the device addresses it (nullptr: none).
std::atomic<int*> g_sink{nullptr};

int setup(DeviceOnce* table, cudaError_t (*fn)()) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CFA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return CFA_ERR_CUDA;
  DeviceOnce& d = table[dev];
  std::call_once(d.flag, [&] { d.result = fn(); });
  return d.result == cudaSuccess ? CFA_OK : CFA_ERR_LAUNCH;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool strides_ok(const int64_t* s) {
  return s[0] % 4 == 0 && s[1] % 4 == 0 && s[2] % 4 == 0;
}

bool head_dim_ok(int64_t D, bool any_dim) {
  return any_dim ? (D == 32 || D == 64 || D == 128) : D == CFA_HEAD_DIM;
}

// Common shape checks. Returns CFA_OK with *empty set when there is nothing to do. any_dim: the
// head-dim-generic entry points (32, 64, 128); otherwise the reference's gate (64 only).
int check_dims(int64_t B, int64_t H, int64_t S, int64_t D, bool any_dim, bool* empty) {
  *empty = false;
  if (B < 0 || H < 0 || S < 0 || D < 0) return CFA_ERR_SHAPE;
  if (!head_dim_ok(D, any_dim)) return CFA_ERR_HEAD_DIM;
  if (B == 0 || H == 0 || S == 0) {
    *empty = true;
    return CFA_OK;
  }
  // Kernel indices: (b * H + h) and its tiles fit int32; element offsets are int64.
  const int64_t lim = (int64_t(1) << 31) - 1;
  if (B > lim || H > lim || S > lim) return CFA_ERR_OVERFLOW;
  if (B * H > lim / ((S + 31) / 32)) return CFA_ERR_OVERFLOW;  // grid size (smallest tile: 32)
  if (B * H * S > lim) return CFA_ERR_OVERFLOW;                 // row index of L, D
  return CFA_OK;
}

int fwd_impl(const float* q, const int64_t q_strides[3], const float* k,
             const int64_t k_strides[3], const float* v, const int64_t v_strides[3], float* o,
             float* lse, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, float scale,
             int causal, void* stream, bool any_dim, Pair pair) {
  bool empty = false;
  int st = check_dims(batch, heads, seq, head_dim, any_dim, &empty);
  if (st != CFA_OK || empty) return st;
  if (!q || !k || !v || !o || !lse || !q_strides || !k_strides || !v_strides) return CFA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return CFA_ERR_ALIGNMENT;
  if (!strides_ok(q_strides) || !strides_ok(k_strides) || !strides_ok(v_strides))
    return CFA_ERR_ALIGNMENT;
  const bool d64 = head_dim == 64;
  // The tensor-core pair takes head dims 64 and 32; 128 runs on the CUDA-core kernels.
  const bool tc = (d64 || head_dim == 32) && pair == Pair::kTensorCore;
  st = tc    ? setup(g_fwd_tc_once, cfa::setup_fwd_tc_attributes)
       : d64 ? setup(g_fwd_once, cfa::setup_fwd_attributes)
             : setup(g_hd_once, cfa::setup_hd_attributes);
  if (st != CFA_OK) return st;

  FwdArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.o = o;
  a.lse = lse;
  a.q_sb = q_strides[0];
  a.q_sh = q_strides[1];
  a.q_ss = q_strides[2];
  a.k_sb = k_strides[0];
  a.k_sh = k_strides[1];
  a.k_ss = k_strides[2];
  a.v_sb = v_strides[0];
  a.v_sh = v_strides[1];
  a.v_ss = v_strides[2];
  a.B = static_cast<int>(batch);
  a.H = static_cast<int>(heads);
  a.S = static_cast<int>(seq);
  a.scale = scale;
  a.sink = g_sink.load(std::memory_order_relaxed);
  const int bm = d64 ? cfa::fwd_tile_rows(seq) : cfa::hd_fwd_rows(static_cast<int>(head_dim), seq);
  a.n_qtiles = static_cast<int>((seq + bm - 1) / bm);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = tc    ? cfa::launch_fwd_tc(a, static_cast<int>(head_dim), causal != 0, s)
                        : d64 ? cfa::launch_fwd(a, causal != 0, s)
                              : cfa::launch_hd_fwd(a, static_cast<int>(head_dim), causal != 0, s);
  return e == cudaSuccess ? CFA_OK : CFA_ERR_LAUNCH;
}

int bwd_impl(const float* q, const int64_t q_strides[3], const float* k,
             const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
             const float* o, const float* lse, const float* d_o, const int64_t do_strides[3],
             float* dqkv, void* workspace, size_t workspace_bytes, int64_t batch, int64_t heads,
             int64_t seq, int64_t head_dim, float scale, int causal, void* stream, bool any_dim,
             Pair pair) {
  bool empty = false;
  int st = check_dims(batch, heads, seq, head_dim, any_dim, &empty);
  if (st != CFA_OK || empty) return st;
  if (!q || !k || !v || !o || !lse || !d_o || !dqkv || !workspace || !q_strides || !k_strides ||
      !v_strides || !do_strides)
    return CFA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(d_o) ||
      !aligned16(dqkv))
    return CFA_ERR_ALIGNMENT;
  if (!strides_ok(q_strides) || !strides_ok(k_strides) || !strides_ok(v_strides) ||
      !strides_ok(do_strides))
    return CFA_ERR_ALIGNMENT;
  const cfa::BwdWorkspace lay = cfa::bwd_workspace_layout(batch, heads, seq, head_dim);
  if (workspace_bytes < lay.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return CFA_ERR_WORKSPACE;
  const bool d64 = head_dim == 64;
  // The tensor-core backward pairs with the tensor-core forward (the scores it recomputes are the
  // forward's, bit for bit), at every length: its dQ takes the no-wait partials when the
  // workspace holds them, else the turn chain (the same sums, bit for bit).
  const bool tc = (d64 || head_dim == 32) && pair == Pair::kTensorCore;
  st = tc    ? setup(g_bwd_tc_once, cfa::setup_bwd_tc_attributes)
       : d64 ? setup(g_bwd_once, cfa::setup_bwd_attributes)
             : setup(g_hd_once, cfa::setup_hd_attributes);
  if (st != CFA_OK) return st;

  char* ws = static_cast<char*>(workspace);
  int* ticket = reinterpret_cast<int*>(ws + lay.ticket_off);
  int* turn = reinterpret_cast<int*>(ws + lay.turn_off);
  float* dsum = reinterpret_cast<float*>(ws + lay.dsum_off);
  const int nqt = static_cast<int>((seq + cfa::BWD_BM - 1) / cfa::BWD_BM);
  const int nkb = static_cast<int>((seq + cfa::BWD_BN - 1) / cfa::BWD_BN);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);

  PrepArgs p;
  p.o = o;
  p.d_o = d_o;
  p.dsum = dsum;
  // ticket and error flag are the first two ints; the turn counters start at turn_off. Clear
  // the header and the counters as one range.
  p.zero = ticket;
  p.n_zero = static_cast<int64_t>(lay.turn_off / sizeof(int)) + batch * heads * nqt;
  p.do_sb = do_strides[0];
  p.do_sh = do_strides[1];
  p.do_ss = do_strides[2];
  p.B = static_cast<int>(batch);
  p.H = static_cast<int>(heads);
  p.S = static_cast<int>(seq);
  cudaError_t e = d64 ? cfa::launch_bwd_prep(p, s)
                      : cfa::launch_hd_bwd_prep(p, static_cast<int>(head_dim), s);
  if (e != cudaSuccess) return CFA_ERR_LAUNCH;

  BwdArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.d_o = d_o;
  a.lse = lse;
  a.dsum = dsum;
  a.dqkv = dqkv;
  a.turn = turn;
  a.ticket = ticket;
  a.err = ticket + 1;
  a.q_sb = q_strides[0];
  a.q_sh = q_strides[1];
  a.q_ss = q_strides[2];
  a.k_sb = k_strides[0];
  a.k_sh = k_strides[1];
  a.k_ss = k_strides[2];
  a.v_sb = v_strides[0];
  a.v_sh = v_strides[1];
  a.v_ss = v_strides[2];
  a.do_sb = do_strides[0];
  a.do_sh = do_strides[1];
  a.do_ss = do_strides[2];
  a.B = static_cast<int>(batch);
  a.H = static_cast<int>(heads);
  a.S = static_cast<int>(seq);
  a.scale = scale;
  a.n_qtiles = nqt;
  a.n_kblocks = nkb;
  a.timeout_ns = cfa::WAIT_TIMEOUT_NS;
  a.sink = g_sink.load(std::memory_order_relaxed);
  // The no-wait dQ path when the workspace holds the partials (same results, bit for bit).
  a.dq_part = (lay.total_fast > lay.total && workspace_bytes >= lay.total_fast)
                  ? reinterpret_cast<float*>(ws + lay.part_off)
                  : nullptr;
  e = tc    ? cfa::launch_bwd_tc(a, static_cast<int>(head_dim), causal != 0, s)
      : d64 ? cfa::launch_bwd(a, causal != 0, s)
            : cfa::launch_hd_bwd(a, static_cast<int>(head_dim), causal != 0, s);
  return e == cudaSuccess ? CFA_OK : CFA_ERR_LAUNCH;
}

}  // namespace

namespace cfa {
int* error_sink() { return g_sink.load(std::memory_order_relaxed); }
}  // namespace cfa

extern "C" {

int cfa_abi_version(void) { return (2 << 16) | 2; }

const char* cfa_strerror(int status) {
  switch (status) {
    case CFA_OK: return "fused_attention: ok";
    case CFA_ERR_HEAD_DIM:
      return "fused_attention: the CUDA kernels take head_dim 64 (cfa_*_f32: 32, 64 or 128)";
    case CFA_ERR_ALIGNMENT: return "fused_attention: rows must be 16-byte aligned";
    case CFA_ERR_SHAPE: return "fused_attention: negative dimension";
    case CFA_ERR_OVERFLOW: return "fused_attention: problem size exceeds the kernels' index range";
    case CFA_ERR_NULL: return "fused_attention: null pointer";
    case CFA_ERR_WORKSPACE: return "fused_attention: workspace too small or misaligned";
    case CFA_ERR_LAUNCH: return "fused_attention: kernel launch failed";
    case CFA_ERR_TIMEOUT: return "fused_attention: a bounded device wait expired (results invalid)";
    case CFA_ERR_CUDA: return "fused_attention: CUDA runtime error";
    default: return "fused_attention: unknown status";
  }
}

int cfa_fwd_f32_d64(const float* q, const int64_t q_strides[3], const float* k,
                    const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
                    float* o, float* lse, int64_t batch, int64_t heads, int64_t seq,
                    int64_t head_dim, float scale, int causal, void* stream) {
  return fwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, batch, heads, seq, head_dim,
                  scale, causal, stream, false, Pair::kTensorCore);
}

int cfa_fwd_f32_d64_ffma(const float* q, const int64_t q_strides[3], const float* k,
                         const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
                         float* o, float* lse, int64_t batch, int64_t heads, int64_t seq,
                         int64_t head_dim, float scale, int causal, void* stream) {
  return fwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, batch, heads, seq, head_dim,
                  scale, causal, stream, false, Pair::kFfma);
}

int cfa_fwd_f32(const float* q, const int64_t q_strides[3], const float* k,
                const int64_t k_strides[3], const float* v, const int64_t v_strides[3], float* o,
                float* lse, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                float scale, int causal, void* stream) {
  return fwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, batch, heads, seq, head_dim,
                  scale, causal, stream, true, Pair::kTensorCore);
}

size_t cfa_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 256;
  return cfa::bwd_workspace_layout(batch, heads, seq).total;
}

size_t cfa_bwd_workspace_bytes_fast(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 256;
  return cfa::bwd_workspace_layout(batch, heads, seq).total_fast;
}

size_t cfa_bwd_workspace_bytes_hd(int64_t batch, int64_t heads, int64_t seq, int64_t head_dim) {
  if (batch <= 0 || heads <= 0 || seq <= 0 || !head_dim_ok(head_dim, true)) return 256;
  return cfa::bwd_workspace_layout(batch, heads, seq, head_dim).total;
}

size_t cfa_bwd_workspace_bytes_fast_hd(int64_t batch, int64_t heads, int64_t seq,
                                       int64_t head_dim) {
  if (batch <= 0 || heads <= 0 || seq <= 0 || !head_dim_ok(head_dim, true)) return 256;
  return cfa::bwd_workspace_layout(batch, heads, seq, head_dim).total_fast;
}

int cfa_bwd_f32_d64(const float* q, const int64_t q_strides[3], const float* k,
                    const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
                    const float* o, const float* lse, const float* d_o,
                    const int64_t do_strides[3], float* dqkv, void* workspace,
                    size_t workspace_bytes, int64_t batch, int64_t heads, int64_t seq,
                    int64_t head_dim, float scale, int causal, void* stream) {
  return bwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, d_o, do_strides, dqkv,
                  workspace, workspace_bytes, batch, heads, seq, head_dim, scale, causal, stream,
                  false, Pair::kTensorCore);
}

int cfa_bwd_f32_d64_ffma(const float* q, const int64_t q_strides[3], const float* k,
                         const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
                         const float* o, const float* lse, const float* d_o,
                         const int64_t do_strides[3], float* dqkv, void* workspace,
                         size_t workspace_bytes, int64_t batch, int64_t heads, int64_t seq,
                         int64_t head_dim, float scale, int causal, void* stream) {
  return bwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, d_o, do_strides, dqkv,
                  workspace, workspace_bytes, batch, heads, seq, head_dim, scale, causal, stream,
                  false, Pair::kFfma);
}

int cfa_fwd_f32_ffma(const float* q, const int64_t q_strides[3], const float* k,
                     const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
                     float* o, float* lse, int64_t batch, int64_t heads, int64_t seq,
                     int64_t head_dim, float scale, int causal, void* stream) {
  return fwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, batch, heads, seq, head_dim,
                  scale, causal, stream, true, Pair::kFfma);
}

int cfa_bwd_f32_ffma(const float* q, const int64_t q_strides[3], const float* k,
                     const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
                     const float* o, const float* lse, const float* d_o,
                     const int64_t do_strides[3], float* dqkv, void* workspace,
                     size_t workspace_bytes, int64_t batch, int64_t heads, int64_t seq,
                     int64_t head_dim, float scale, int causal, void* stream) {
  return bwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, d_o, do_strides, dqkv,
                  workspace, workspace_bytes, batch, heads, seq, head_dim, scale, causal, stream,
                  true, Pair::kFfma);
}

int cfa_bwd_f32(const float* q, const int64_t q_strides[3], const float* k,
                const int64_t k_strides[3], const float* v, const int64_t v_strides[3],
                const float* o, const float* lse, const float* d_o, const int64_t do_strides[3],
                float* dqkv, void* workspace, size_t workspace_bytes, int64_t batch,
                int64_t heads, int64_t seq, int64_t head_dim, float scale, int causal,
                void* stream) {
  return bwd_impl(q, q_strides, k, k_strides, v, v_strides, o, lse, d_o, do_strides, dqkv,
                  workspace, workspace_bytes, batch, heads, seq, head_dim, scale, causal, stream,
                  true, Pair::kTensorCore);
}

// The projection GEMM: any strides for A and B (the split pass gathers them; K-contiguous rows
// that are 16-byte aligned are read 16 bytes at a time), 16-byte rows for C.
namespace {
DeviceOnce g_linear_once[kMaxDevices];

// M, N and K up to 2^30: every tile, chunk and K index the kernels form fits int32.
constexpr int64_t kLinMax = int64_t(1) << 30;
}  // namespace

size_t cfa_matmul_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0 || m > kLinMax || n > kLinMax || k > kLinMax) return 0;
  return cfa::linear_plan(m, n, k).ws_bytes;
}

int cfa_matmul_f32(const float* a, int64_t a_row_stride, int64_t a_col_stride, const float* b,
                   int64_t b_row_stride, int64_t b_col_stride, float* c, int64_t c_row_stride,
                   int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (m < 0 || n < 0 || k < 0) return CFA_ERR_SHAPE;
  if (m == 0 || n == 0) return CFA_OK;
  if (m > kLinMax || n > kLinMax || k > kLinMax) return CFA_ERR_OVERFLOW;
  if (!c || (k > 0 && (!a || !b || !workspace))) return CFA_ERR_NULL;
  if (!aligned16(c) || (m > 1 && c_row_stride % 4 != 0)) return CFA_ERR_ALIGNMENT;
  cfa::LinArgs args{};
  cfa::LinPlan p{};
  if (k > 0) {
    p = cfa::linear_plan(m, n, k);
    if (workspace_bytes < p.ws_bytes) return CFA_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return CFA_ERR_WORKSPACE;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    args.pa = ws + p.pa_off;
    args.pb = ws + p.pb_off;
    args.part = reinterpret_cast<float*>(ws + p.part_off);
    args.a_k_contig = a_col_stride == 1;
    args.b_k_contig = b_row_stride == 1;
    args.a_vec = args.a_k_contig && aligned16(a) && (m == 1 || a_row_stride % 4 == 0);
    args.b_vec = args.b_k_contig && aligned16(b) && (n == 1 || b_col_stride % 4 == 0);
  }
  const int st = setup(g_linear_once, cfa::setup_linear_attributes);
  if (st != CFA_OK) return st;
  args.a = a;
  args.a_sm = a_row_stride;
  args.a_sk = a_col_stride;
  args.b = b;
  args.b_sk = b_row_stride;
  args.b_sn = b_col_stride;
  args.c = c;
  args.c_sm = c_row_stride;
  args.M = static_cast<int>(m);
  args.N = static_cast<int>(n);
  args.K = static_cast<int>(k);
  args.tiles_m = p.tiles_m;
  args.tiles_n = p.tiles_n;
  args.ksplit = p.ksplit;
  args.chunk_steps = p.chunk_steps;
  args.nks = p.nks;
  args.ldp = p.ldp;
  args.sink = g_sink.load(std::memory_order_relaxed);
  const cudaError_t e = cfa::launch_linear_tc(args, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CFA_OK : CFA_ERR_LAUNCH;
}

int cfa_matmul_status(void* stream) {
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return CFA_ERR_CUDA;
  int flag = 0;
  if (cfa::linear_status(&flag) != cudaSuccess) return CFA_ERR_CUDA;
  return flag != 0 ? CFA_ERR_TIMEOUT : CFA_OK;
}

int cfa_selftest_bounded_wait(void* workspace, int64_t timeout_ns, int blocks, void* stream) {
  if (!workspace) return CFA_ERR_NULL;
  if (timeout_ns <= 0 || timeout_ns > 10000000000ll || blocks < 1 || blocks > 1024)
    return CFA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return CFA_ERR_WORKSPACE;
  const cudaError_t e = cfa::launch_selftest_wait(static_cast<int*>(workspace),
                                                  static_cast<uint64_t>(timeout_ns), blocks,
                                                  g_sink.load(std::memory_order_relaxed),
                                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CFA_OK : CFA_ERR_LAUNCH;
}

int cfa_error_sink(int* host_flag) {
  if (host_flag == nullptr) {
    g_sink.store(nullptr);
    return CFA_OK;
  }
  if ((reinterpret_cast<uintptr_t>(host_flag) & 3u) != 0) return CFA_ERR_ALIGNMENT;
  // Only page-locked host memory the device can address is accepted: a kernel's store to anything
  // else would fault.
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, host_flag) != cudaSuccess) return CFA_ERR_CUDA;
  if (attr.type != cudaMemoryTypeHost) return CFA_ERR_CUDA;
  void* dev_ptr = nullptr;
  if (cudaHostGetDevicePointer(&dev_ptr, host_flag, 0) != cudaSuccess || dev_ptr == nullptr)
    return CFA_ERR_CUDA;
  g_sink.store(static_cast<int*>(dev_ptr));
  return CFA_OK;
}

int cfa_fwd_status(void* stream) {
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return CFA_ERR_CUDA;
  int flag = 0;
  if (cfa::fwd_tc_status(&flag) != cudaSuccess) return CFA_ERR_CUDA;
  return flag != 0 ? CFA_ERR_TIMEOUT : CFA_OK;
}

int cfa_bwd_status(const void* workspace, void* stream) {
  if (!workspace) return CFA_ERR_NULL;
  int flags[2] = {0, 0};
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(flags, workspace, sizeof(flags), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return CFA_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return CFA_ERR_CUDA;
  return flags[1] != 0 ? flags[1] : CFA_OK;
}

}  // extern "C"
