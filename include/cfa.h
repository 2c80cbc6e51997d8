/* SPDX-License-Identifier: MIT OR Apache-2.0
 *
 * cfa.h -- the C ABI of the B200 (sm_100a) fused fp32 attention, head_dim 64.
 *
 * This is the drop-in boundary under candle-fused-attn's public API. The Rust crate's launch layer
 * (`src/cuda.rs`) loads a PTX module and launches three kernels with fixed argument lists; these
 * entry points replace that layer one for one, so the crate's `src/lib.rs` (alignment gate, qkv
 * geometry, saved log-sum-exp, candle CustomOp glue) stays as it is and only swaps its two calls:
 *
 *   cfa_fwd_f32_d64            replaces  cuda::forward   (src/cuda.rs:140-185), which launched
 *                                        fattn_fwd_f32_d64 (kernels/fused_attn.cu:469-475)
 *   cfa_bwd_workspace_bytes    replaces  the three `dev.alloc` calls of cuda::backward
 *                                        (src/cuda.rs:203-209): D, the dQ turn counters
 *   cfa_bwd_f32_d64            replaces  cuda::backward  (src/cuda.rs:190-260), which launched
 *                                        fattn_bwd_dot_f32_d64 (kernels/fused_attn.cu:45-48) and
 *                                        fattn_bwd_f32_d64 (kernels/fused_attn.cu:213-221)
 *   cfa_bwd_status             has no kernel counterpart: reads the device error flag that the
 *                                        bounded waits of the backward set (the reference spins
 *                                        without a bound, kernels/fused_attn.cu:161-170)
 *   cfa_strerror               replaces  the `Error::Msg` strings of src/cuda.rs:69-93
 *   cfa_fwd_f32, cfa_bwd_f32,  extend     the above to head dims 32 and 128, which the
 *   cfa_bwd_workspace_bytes*_hd            reference's CUDA path rejects (src/cuda.rs:85-93) and
 *                                          lists as later work (ROADMAP.md "head_dim 32 and 128");
 *                                          its CPU path (src/lib.rs:241-299) takes any head dim
 *   cfa_error_sink             has no counterpart: a host-visible flag that every bounded-wait
 *                                          expiry reaches without a synchronisation
 *   cfa_matmul_f32,            the projection next to the path: candle's broadcast_matmul of
 *   cfa_matmul_workspace_bytes           the training step (examples/tutorial.rs:103-118) as a
 *   cfa_matmul_status                    tensor-core kernel
 *
 * Head dim 64 runs one kernel pair, as the reference does (src/cuda.rs:140-260): the tensor-core
 * pair (csrc/fwd_tc.cu, csrc/bwd_tc.cu). A backward must run on the forward's L of the same pair
 * (it recomputes the forward's scores bit for bit); the entry points fix the pair, so there is
 * no process-wide setting two users could disagree on. The CUDA-core pair stays available under
 * its own names (cfa_fwd_f32_d64_ffma, cfa_bwd_f32_d64_ffma; cfa_fwd_f32_ffma, cfa_bwd_f32_ffma
 * at every head dim) for comparison.
 *
 * Conventions (the reference's, src/cuda.rs:60-67 and src/lib.rs:165-188):
 *  - Every pointer is a device pointer at the operand's first element, on the current device.
 *  - A [b, h, s, d] operand is described by its (batch, head, seq) strides in floats; d is
 *    contiguous. Pointers and strides must be multiples of 4 floats (16-byte rows), which the
 *    caller establishes (src/lib.rs:112, :165-168); violations return CFA_ERR_ALIGNMENT.
 *  - Outputs are dense: O [b, s, h, 64] (merge-heads layout), L [b, h, s],
 *    dqkv [b, s, 3, h, 64] (dQ, dK, dV interleaved: a fused qkv projection's gradient).
 *  - Everything is asynchronous on `stream` (a cudaStream_t; NULL = the legacy default stream).
 *    No entry point allocates memory or keeps state besides a once-per-device kernel attribute
 *    set-up and the registered error sink; only the *_status queries synchronise. Calls on
 *    different streams may run concurrently.
 *  - Zero batch, heads or seq is a valid empty problem: CFA_OK and nothing is launched (the
 *    reference panics there, its audit item B2).
 *  - Results are bit-identical across reruns and independent of the GPU's SM count and of how
 *    the batch is split over GPUs.
 */
#ifndef CFA_H
#define CFA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CFA_HEAD_DIM 64 /* src/lib.rs:91 CUDA_HEAD_DIM */

enum cfa_status {
  CFA_OK = 0,
  CFA_ERR_HEAD_DIM = 1,   /* head_dim != 64 (src/cuda.rs:85-93) */
  CFA_ERR_ALIGNMENT = 2,  /* a pointer or stride is not a multiple of 4 floats */
  CFA_ERR_SHAPE = 3,      /* a negative dimension */
  CFA_ERR_OVERFLOW = 4,   /* an index or grid size past the kernels' 32/64-bit range */
  CFA_ERR_NULL = 5,       /* a null pointer for a non-empty problem */
  CFA_ERR_WORKSPACE = 6,  /* workspace smaller than cfa_bwd_workspace_bytes or misaligned */
  CFA_ERR_LAUNCH = 7,     /* the CUDA launch failed */
  CFA_ERR_TIMEOUT = 8,    /* a bounded device-side wait of a kernel expired */
  CFA_ERR_CUDA = 9        /* another CUDA runtime error (device query, copy, sync) */
};

/* Forward: O = softmax(q k^T * scale [+ causal mask]) v and L = rowwise log-sum-exp.
 * q, k, v: [batch, heads, seq, 64] through (batch, head, seq) strides `*_strides[3]`.
 * o: [batch, seq, heads, 64] dense.  lse: [batch, heads, seq] dense.
 * Replaces src/cuda.rs:140-185 (launch of kernels/fused_attn.cu:469). */
int cfa_fwd_f32_d64(const float* q, const int64_t q_strides[3],
                    const float* k, const int64_t k_strides[3],
                    const float* v, const int64_t v_strides[3],
                    float* o, float* lse,
                    int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                    float scale, int causal, void* stream);

/* Bytes of device scratch the backward needs (D = rowsum(dO o O), the dQ turn counters, a work
 * ticket and the error flag). The caller allocates it (256-byte aligned); its contents need no
 * initialisation. Replaces the allocations at src/cuda.rs:203-209. */
size_t cfa_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq);

/* Bytes of device scratch that let the backward skip the waits of its dQ key-block chain: with
 * at least this much workspace, each key block stores its dQ partials to the scratch and the
 * last block of a (batch, head) to finish adds them in key-block order -- the same sums, bit for
 * bit, as with cfa_bwd_workspace_bytes, in less time. Applies to seq <= 1024 (at most 16 key
 * blocks of 64; the partials take ceil(seq / 64) times the size of dQ); for longer sequences it
 * equals cfa_bwd_workspace_bytes. Canvas b64 h6 s240: 94.7 MB. */
size_t cfa_bwd_workspace_bytes_fast(int64_t batch, int64_t heads, int64_t seq);

/* Backward from dO to one dqkv [batch, seq, 3, heads, 64] buffer (dQ, dK, dV interleaved).
 * o, lse: the forward's outputs (dense, as cfa_fwd_f32_d64 writes them).
 * d_o: [batch, heads, seq, 64] through `do_strides[3]`.
 * dQ is summed over key blocks in key-block order, so reruns are bit-identical.
 * Replaces src/cuda.rs:190-260 (launches of kernels/fused_attn.cu:45 and :213). */
int cfa_bwd_f32_d64(const float* q, const int64_t q_strides[3],
                    const float* k, const int64_t k_strides[3],
                    const float* v, const int64_t v_strides[3],
                    const float* o, const float* lse,
                    const float* d_o, const int64_t do_strides[3],
                    float* dqkv, void* workspace, size_t workspace_bytes,
                    int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                    float scale, int causal, void* stream);

/* Head dims 32, 64 and 128 (no counterpart in the reference's CUDA path, which takes 64 only).
 * The same arguments, layouts (with 64 replaced by head_dim), orders of summation and results as
 * the _d64 entry points; for head_dim 64 they ARE those entry points. Head dims 64 and 32 run the
 * tensor-core pair (32: the head-dim-64 kernels on rows zero-filled past the head dim, the
 * all-zero K-steps skipped), 128 the CUDA-core kernels of csrc/hd_ffma.cu. Any other head_dim
 * returns CFA_ERR_HEAD_DIM. Workspace sizes take the head dim because the dQ partials hold
 * head_dim floats per row (the rest of the workspace does not depend on it). */
int cfa_fwd_f32(const float* q, const int64_t q_strides[3],
                const float* k, const int64_t k_strides[3],
                const float* v, const int64_t v_strides[3],
                float* o, float* lse,
                int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                float scale, int causal, void* stream);

size_t cfa_bwd_workspace_bytes_hd(int64_t batch, int64_t heads, int64_t seq, int64_t head_dim);

size_t cfa_bwd_workspace_bytes_fast_hd(int64_t batch, int64_t heads, int64_t seq,
                                       int64_t head_dim);

int cfa_bwd_f32(const float* q, const int64_t q_strides[3],
                const float* k, const int64_t k_strides[3],
                const float* v, const int64_t v_strides[3],
                const float* o, const float* lse,
                const float* d_o, const int64_t do_strides[3],
                float* dqkv, void* workspace, size_t workspace_bytes,
                int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                float scale, int causal, void* stream);

/* The CUDA-core (FFMA) pair at head dim 64: the same arguments, layouts and contract as
 * cfa_fwd_f32_d64 / cfa_bwd_f32_d64, computed with packed fp32 FMAs (csrc/fwd_ffma.cu,
 * csrc/bwd_ffma.cu). Pair cfa_bwd_f32_d64_ffma only with the L of cfa_fwd_f32_d64_ffma (and the
 * tensor-core backward only with the tensor-core forward's L): across pairs the recomputed scores
 * round differently and the gradients drift up to 1.4x past the reference's 5e-6 band. No
 * counterpart in the reference (one kernel pair). */
int cfa_fwd_f32_d64_ffma(const float* q, const int64_t q_strides[3],
                         const float* k, const int64_t k_strides[3],
                         const float* v, const int64_t v_strides[3],
                         float* o, float* lse,
                         int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                         float scale, int causal, void* stream);

int cfa_bwd_f32_d64_ffma(const float* q, const int64_t q_strides[3],
                         const float* k, const int64_t k_strides[3],
                         const float* v, const int64_t v_strides[3],
                         const float* o, const float* lse,
                         const float* d_o, const int64_t do_strides[3],
                         float* dqkv, void* workspace, size_t workspace_bytes,
                         int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                         float scale, int causal, void* stream);

/* The CUDA-core pair at head dims 32, 64 and 128 (the cfa_fwd_f32 / cfa_bwd_f32 contract): for 64
 * the _d64_ffma entry points, for 32 and 128 csrc/hd_ffma.cu. At 128 it is what cfa_fwd_f32 runs;
 * at 32 it stays for comparison with the tensor-core pair. The same pairing rule applies. */
int cfa_fwd_f32_ffma(const float* q, const int64_t q_strides[3],
                     const float* k, const int64_t k_strides[3],
                     const float* v, const int64_t v_strides[3],
                     float* o, float* lse,
                     int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                     float scale, int causal, void* stream);

int cfa_bwd_f32_ffma(const float* q, const int64_t q_strides[3],
                     const float* k, const int64_t k_strides[3],
                     const float* v, const int64_t v_strides[3],
                     const float* o, const float* lse,
                     const float* d_o, const int64_t do_strides[3],
                     float* dqkv, void* workspace, size_t workspace_bytes,
                     int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                     float scale, int causal, void* stream);

/* Size of the static scratch of cfa_bwd_f32_d64_noalloc (4 MiB per GPU that loads the library). */
#define CFA_NOALLOC_SCRATCH_BYTES (4u << 20)

/* The backward without any allocation, for callers that cannot call cudaMalloc (a host framework
 * whose allocator owns all device memory, a real-time loop that cannot risk an allocation, an FFI
 * that passes only the tensors it was given).
 * Same arguments and results as cfa_bwd_f32_d64 minus the workspace: the scratch is a file-scope
 * static device array of CFA_NOALLOC_SCRATCH_BYTES, held by every GPU that loads the library
 * until exit. Has no counterpart in the reference (its launch layer always allocates,
 * src/cuda.rs:203-209).
 *  - Problems needing more scratch than that (cfa_bwd_workspace_bytes > 4 MiB) return
 *    CFA_ERR_WORKSPACE before anything runs.
 *  - Other bad arguments (head dim, negative or oversized dimensions, null pointers) return the
 *    codes cfa_bwd_f32_d64 returns for them, checked before the scratch size.
 *  - The first call on a device looks up the array's device address and caches it; a failed
 *    lookup returns CFA_ERR_CUDA, then and on every later call on that device. The cached
 *    address stays valid until the device's primary context is destroyed: do not call this
 *    entry point on a device after cudaDeviceReset.
 *  - All calls on a device share the array (each call resets what must start at zero); calls
 *    that can overlap on the GPU race and must be ordered by the caller.
 *  - cfa_bwd_noalloc_status reads the array's error flag. */
int cfa_bwd_f32_d64_noalloc(const float* q, const int64_t q_strides[3],
                            const float* k, const int64_t k_strides[3],
                            const float* v, const int64_t v_strides[3],
                            const float* o, const float* lse,
                            const float* d_o, const int64_t do_strides[3],
                            float* dqkv,
                            int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                            float scale, int causal, void* stream);

/* cfa_bwd_status for the static scratch of cfa_bwd_f32_d64_noalloc on the current device:
 * synchronises `stream` and returns CFA_ERR_TIMEOUT if a bounded wait of the last no-allocation
 * backward on this device expired, else CFA_OK (CFA_ERR_CUDA if the array cannot be addressed).
 * Has no counterpart in the reference. */
int cfa_bwd_noalloc_status(void* stream);

/* Synchronises `stream` and returns CFA_ERR_TIMEOUT if a bounded wait of the last backward that
 * used `workspace` expired (its results are then invalid), else CFA_OK (or CFA_ERR_CUDA). */
int cfa_bwd_status(const void* workspace, void* stream);

/* Synchronises `stream` and returns CFA_ERR_TIMEOUT if a bounded wait of a tensor-core forward
 * since the last call expired (its outputs are then invalid), else CFA_OK; clears the flag. */
int cfa_fwd_status(void* stream);

/* Self-test of the failure detection (no counterpart in the reference, whose spin has no bound):
 * launches `blocks` blocks whose waits -- the bounded routine of the backward's dQ chain -- can
 * never be satisfied. Block 0 gives up after `timeout_ns`, the others bail out as soon as it has
 * flagged the error, so the kernel ends after about `timeout_ns`, leaving CFA_ERR_TIMEOUT in the
 * 256-byte, 256-aligned `workspace` for cfa_bwd_status to read. No GPU fault, no hang. */
int cfa_selftest_bounded_wait(void* workspace, int64_t timeout_ns, int blocks, void* stream);

/* Registers a host-visible error flag (NULL unregisters; the default is none). `host_flag` must
 * be page-locked host memory the GPUs can address (cudaHostAlloc, cudaMallocHost, or a pinned
 * tensor), 4-byte aligned; anything else returns CFA_ERR_CUDA (CFA_ERR_ALIGNMENT if misaligned)
 * and leaves the registration unchanged. Every kernel launched afterwards (any device, any
 * stream) writes CFA_ERR_TIMEOUT there when one of its bounded waits expires -- as well as into
 * the flags cfa_fwd_status / cfa_bwd_status read -- so the caller learns of an expiry by reading
 * one int, without synchronising; the library never clears it. Process-wide: one flag for all
 * callers, which each see every expiry. The memory must stay valid while kernels launched with
 * it registered can run. Has no counterpart in the reference, whose waits have no bound. */
int cfa_error_sink(int* host_flag);

/* The projection next to the attention: C = A B over fp32 on the tensor cores (three bf16 parts
 * per operand, six products, fp32 sums per 64-element window) -- the contraction of candle's
 * `Tensor::broadcast_matmul` in the reference's training step (examples/tutorial.rs:110: qkv =
 * x W_qkv feeding fused_attention_qkv; the step's gradient of W_qkv is x^T dqkv, tutorial.rs:113).
 * In candle that matmul is cuBLAS SGEMM on the GPU and the gemm crate on the CPU (candle-core's
 * matmul, not in the crate); this entry point is the B200 kernel for it.
 *   A(i, p) = a[i a_row_stride + p a_col_stride], i < m, p < k
 *   B(p, j) = b[p b_row_stride + j b_col_stride], j < n
 *   C(i, j) = c[i c_row_stride + j]
 * A and B may have any strides (x W, dY W^T and x^T dY need no copy; rows with the K stride 1 and
 * 16-byte alignment are read fastest); c and c_row_stride keep C's rows 16-byte aligned (a
 * multiple of 4 floats) -- else CFA_ERR_ALIGNMENT. m, n, k <= 2^30. m or n = 0: CFA_OK, nothing
 * launched; k = 0: C = 0. For k > 0 the call needs cfa_matmul_workspace_bytes(m, n, k) bytes of
 * 256-byte-aligned device workspace: each operand's bf16 parts (6 bytes an element, padded to
 * 128 x 16 blocks) and, when the output has few 128 x 128 tiles and K is cut into chunks, their
 * partial tiles. Bit-identical across reruns and GPUs; asynchronous on `stream`. */
size_t cfa_matmul_workspace_bytes(int64_t m, int64_t n, int64_t k);
int cfa_matmul_f32(const float* a, int64_t a_row_stride, int64_t a_col_stride,
                   const float* b, int64_t b_row_stride, int64_t b_col_stride,
                   float* c, int64_t c_row_stride, int64_t m, int64_t n, int64_t k,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Synchronises `stream` and returns CFA_ERR_TIMEOUT if a bounded wait of a cfa_matmul_f32 kernel
 * since the last call expired (its output is then invalid), else CFA_OK; clears the flag. */
int cfa_matmul_status(void* stream);

/* A static description of a status code. */
const char* cfa_strerror(int status);

/* ABI version: (major << 16) | minor (2.0: one kernel pair per entry point, the error sink;
 * 2.1: the projection GEMM; 2.2: head dim 32 on the tensor cores, the generic CUDA-core pair). */
int cfa_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CFA_H */
