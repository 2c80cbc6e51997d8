// SPDX-License-Identifier: MIT OR Apache-2.0
//
// Internal launch interface between the C ABI (cfa_abi.cu) and the kernel translation units.
// Host-only types; no torch, no candle.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "cfa.h"

namespace cfa {

// The forward's tile: fwd_tile_rows(seq) queries per block (64 or 48, whichever pads fewer rows;
// the results do not depend on it), FWD_BN keys per step.
constexpr int FWD_BN = 64;
int fwd_tile_rows(int64_t seq);
constexpr int FWD_THREADS = 128;

// The backward's tile: BWD_BN keys per block (one key block; fixes dQ's summation order, so it
// depends on nothing but this constant), BWD_BM queries per step (one dQ turn counter each).
constexpr int BWD_BN = 64;
constexpr int BWD_BM = 64;
constexpr int BWD_THREADS = 256;
constexpr int PREP_THREADS = 256;

// Sequences of at most PART_MAX_KBLOCKS key blocks (s <= 1024) can take the backward's no-wait dQ
// path: each key block stores its dQ partials to scratch and the last block of a (batch, head) to
// finish sums them in key-block order (the same sums, bit for bit, as the turn chain). The
// partials take n_kblocks times the size of dQ; longer sequences keep the turn chain.
constexpr int PART_MAX_KBLOCKS = 16;

// A bounded wait gives up after this much GPU time (ns) and flags CFA_ERR_TIMEOUT.
constexpr uint64_t WAIT_TIMEOUT_NS = 2000000000ull;

struct FwdArgs {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  float* lse;
  int64_t q_sb, q_sh, q_ss;
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int B, H, S;
  float scale;
  int n_qtiles;
  int wave_ctas;  // tensor-core forward: blocks resident at once (one per SM); 0: none
  int* sink;      // host-visible error flag (cfa_error_sink) or nullptr
};

struct BwdArgs {
  const float* q;
  const float* k;
  const float* v;
  const float* d_o;
  const float* lse;
  const float* dsum;
  float* dqkv;
  int* turn;      // turn chain: [B * H * n_qtiles]; no-wait path: arrival counter per (b, h)
  int* ticket;
  int* err;
  float* dq_part; // no-wait path: [B * H][n_kblocks][S][D] dQ partials; nullptr: turn chain
  int64_t q_sb, q_sh, q_ss;
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t do_sb, do_sh, do_ss;
  int B, H, S;
  float scale;
  int n_qtiles;  // ceil(S / BWD_BM)
  int n_kblocks; // ceil(S / BWD_BN)
  int wave_ctas;  // tensor-core backward: blocks resident at once (one per SM); 0: none
  uint64_t timeout_ns;
  int* sink;      // host-visible error flag (cfa_error_sink) or nullptr
  // Tensor-core backward, split tail (set by its launcher; tail_parts <= 1: none). The key blocks
  // from tail_base on (tail_units of them, the last partial wave) each run as tail_parts blocks,
  // one per contiguous range of query tiles (the roles by a ticket, helpers first); the helpers
  // leave their tiles' dV, dK windows in tail_win and raise tail_flag, the first part adds them in
  // tile order.
  int tail_base, tail_units, tail_parts;
  float* tail_win;  // [tail_units][query tiles][2][128][D] window sums
  int* tail_flag;   // [tail_units][tail_parts] flags, then the tail's ticket counter (cleared by the
                    // prep kernel)
};

struct PrepArgs {
  const float* o;
  const float* d_o;
  float* dsum;
  int* zero;  // ints cleared before the main backward kernel: ticket, error flag, turn counters
  int64_t n_zero;
  int64_t do_sb, do_sh, do_ss;
  int B, H, S;
};

// Workspace layout of the backward (all offsets 256-byte aligned).
struct BwdWorkspace {
  size_t ticket_off;  // int ticket, int err (first 256 bytes)
  size_t turn_off;    // int turn[B * H * n_qtiles]
  size_t dsum_off;    // float D[B * H * S]
  size_t total;       // bytes of the turn-chain layout
  size_t part_off;    // float partials[B * H * n_kblocks * S * D] (no-wait dQ path)
  size_t total_fast;  // bytes with the partials (== total when the path does not apply)
};

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// D: the head dim (the partials hold D floats per row); the layout is otherwise independent of it.
inline BwdWorkspace bwd_workspace_layout(int64_t B, int64_t H, int64_t S, int64_t D = 64) {
  BwdWorkspace w;
  const int64_t nqt = (S + BWD_BM - 1) / BWD_BM;
  w.ticket_off = 0;
  w.turn_off = 256;
  w.dsum_off = w.turn_off + align256(static_cast<size_t>(B * H * nqt) * sizeof(int));
  w.total = w.dsum_off + align256(static_cast<size_t>(B * H * S) * sizeof(float));
  const int64_t nkb = (S + BWD_BN - 1) / BWD_BN;
  w.part_off = w.total;
  w.total_fast = nkb <= PART_MAX_KBLOCKS
                     ? w.total + static_cast<size_t>(nkb * B * H * S) * D * sizeof(float)
                     : w.total;
  return w;
}

size_t bwd_smem_bytes();

// Launchers (return a cudaError_t from the launch). launch_fwd sets the query-tile count itself.
cudaError_t launch_fwd(const FwdArgs& a, int causal, cudaStream_t stream);
// The tensor-core forward (fwd_tc.cu): 128-query tiles, head dim 64 or 32; sets the query-tile
// count itself.
cudaError_t launch_fwd_tc(const FwdArgs& a, int head_dim, int causal, cudaStream_t stream);
// Reads and clears the tensor-core forward's device error flag (1: an MMA wait expired).
cudaError_t fwd_tc_status(int* flag);
// The tensor-core backward (bwd_tc.cu): 128-key blocks, head dim 64 or 32; dQ by the partials
// (dq_part set) or the turn chain; sets the key-block count itself.
cudaError_t launch_bwd_tc(const BwdArgs& a, int head_dim, int causal, cudaStream_t stream);
cudaError_t launch_bwd_prep(const PrepArgs& a, cudaStream_t stream);
cudaError_t launch_bwd(const BwdArgs& a, int causal, cudaStream_t stream);

// Head dims 32 and 128 (csrc/hd_ffma.cu): the forward's query tile (per sequence length), the attribute
// set-up and the launchers; the backward uses the same 64-key blocks and 64-query tiles as head
// dim 64, so BwdArgs, PrepArgs and the workspace layout carry over.
int hd_fwd_rows(int head_dim, int64_t seq);
cudaError_t setup_hd_attributes();
cudaError_t launch_hd_fwd(const FwdArgs& a, int head_dim, int causal, cudaStream_t stream);
cudaError_t launch_hd_bwd_prep(const PrepArgs& a, int head_dim, cudaStream_t stream);
cudaError_t launch_hd_bwd(const BwdArgs& a, int head_dim, int causal, cudaStream_t stream);

// The projection GEMM (linear_tc.cu): C = A B over fp32 on the tensor cores (split bf16 parts).
// A(m, k) = a[m a_sm + k a_sk], B(k, n) = b[k b_sk + n b_sn] (any strides), C(m, n) = c[m c_sm +
// n] (16-byte rows). A split pass writes each operand's bf16 parts into the workspace, the product
// kernel reads them with bulk copies.
constexpr int LIN_SMS = 148;  // the B200's SM count: fixes the K-chunk count, never read off a device

struct LinPlan {
  int tiles_m, tiles_n;  // 128 x 128 output tiles
  int ksplit;            // K chunks (partial tiles summed in chunk order when > 1)
  int chunk_steps;       // K-steps of 16 per chunk (a multiple of 4)
  int nks;               // K-steps of the split parts (ksplit * chunk_steps; zero past K)
  int ldp;               // row length of the partial tiles (N rounded up to 4)
  size_t pa_off, pb_off, part_off;  // workspace: A's parts, B's parts, the partial tiles
  size_t ws_bytes;                  // workspace bytes in all
};
LinPlan linear_plan(int64_t M, int64_t N, int64_t K);

struct LinArgs {
  const float* a;
  int64_t a_sm, a_sk;
  const float* b;
  int64_t b_sk, b_sn;
  float* c;
  int64_t c_sm;
  unsigned char* pa;  // A's parts: [tiles_m][nks] blocks of 3 x 128 x 16 bf16
  unsigned char* pb;  // B's parts: [tiles_n][nks] blocks
  float* part;        // [ksplit][M][ldp] partial tiles, when ksplit > 1
  int M, N, K;
  int tiles_m, tiles_n, ksplit, chunk_steps, nks, ldp;
  int n_items;  // set by the launcher
  int a_k_contig, b_k_contig;  // the operand's K stride is 1
  int a_vec, b_vec;            // ... and its rows are 16-byte aligned (16-byte loads)
  int* sink;    // host-visible error flag (cfa_error_sink) or nullptr
};
cudaError_t setup_linear_attributes();
cudaError_t launch_linear_tc(const LinArgs& a, cudaStream_t stream);
// Reads and clears the projection kernel's device error flag (1: a wait expired).
cudaError_t linear_status(int* flag);

// The failure-detection self-test (cfa_selftest_bounded_wait).
cudaError_t launch_selftest_wait(int* ws, uint64_t short_ns, int blocks, int* sink,
                                 cudaStream_t stream);

// The host-visible error flag registered with cfa_error_sink (its device address), or nullptr.
int* error_sink();

// One-time per-device attribute set-up (dynamic shared memory limits).
cudaError_t setup_fwd_attributes();
cudaError_t setup_fwd_tc_attributes();
cudaError_t setup_bwd_tc_attributes();
cudaError_t setup_bwd_attributes();

}  // namespace cfa
