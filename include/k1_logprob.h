/*
 * k1_logprob.h -- C ABI of the B200 (sm_100a) K1 primitive: per-row log-prob of a
 * target token, entropy and log-sum-exp over a [rows, vocab] block of logits,
 * forward and backward.
 *
 * Every entry point takes plain device pointers, element counts/strides and a CUDA
 * stream handle (cudaStream_t passed as void*; NULL = legacy default stream).  No
 * entry point allocates device memory; only the k1_ring_status diagnostic synchronises;
 * state kept between calls is limited to cached per-device launch parameters (SM count,
 * resident blocks per kernel) and the ring's timeout word.  The caller owns every
 * output buffer, exactly like the reference's torch binding, whose host functions
 * only write into out-parameters (reference: csrc/fused_logprob.cu:284-458,
 * python/kernel_opt/ops.py:24-30,83).
 *
 * Row layout.  Rows are addressed with two stride levels so that a sliced
 * [B, L', V] view such as logits[:, :-1, :] of a [B, L, V] tensor is one call:
 *     element (r, v) lives at  base + (r / inner_rows) * outer_stride
 *                                   + (r % inner_rows) * inner_stride + v
 * A contiguous [N, V] matrix is inner_rows = N, inner_stride = V (outer_stride is
 * then unused).  The vocabulary axis always has unit stride.  The reference only
 * accepts contiguous logits (csrc/fused_logprob.cu:294,364,414).
 *
 * Targets outside [0, vocab) (for example an ignore index of -100) are accepted
 * and follow the reference kernels: the target logit reads as 0, so
 * logprob = -lse, and the backward adds no one-hot term
 * (csrc/fused_logprob.cu:179-185, 279).
 *
 * Return value: K1_OK (0) or a k1_status code; k1_last_error() then returns a
 * message for the calling thread.  Kernel launch errors are reported the same way
 * (the reference does not check launches).
 */
#ifndef K1_LOGPROB_H
#define K1_LOGPROB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 1: initial entry points; 2: adds the scaled forward and backward. */
#define K1_ABI_VERSION 2

/* Element type of logits and d_logits.  Outputs and saved rows are always fp32. */
typedef enum k1_dtype {
    K1_DTYPE_F32 = 0,
    K1_DTYPE_F16 = 1,
    K1_DTYPE_BF16 = 2
} k1_dtype;

typedef enum k1_status {
    K1_OK = 0,
    K1_ERR_INVALID_ARGUMENT = 1, /* bad size, stride, pointer or alignment */
    K1_ERR_UNSUPPORTED_DTYPE = 2,
    K1_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required */
    K1_ERR_CUDA = 4              /* a CUDA runtime call or kernel launch failed */
} k1_status;

/*
 * Per-row partial state of one vocabulary shard (vocab-parallel mode).  Relative to
 * the shard's own maximum m:  z = sum_v exp(x_v - m),  t = sum_v exp(x_v - m)(x_v - m).
 * x_t is the target logit when the target column lies in this shard (has_target = 1).
 * A shard whose columns are all -inf has m = -inf and z = t = 0.
 * No counterpart in the reference (it has no multi-GPU path); the combine rule is the
 * reference's (m, Z, T) merge (csrc/fused_logprob.cu:119-154) carried in fp64.
 */
typedef struct k1_partial {
    double z;
    double t;
    float m;
    float x_t;
    int32_t has_target;
    int32_t reserved;
} k1_partial;

/* Message describing the last failing call made by this thread ("" if none). */
const char* k1_last_error(void);

/* K1_ABI_VERSION of the loaded library. */
int k1_abi_version(void);

/*
 * Diagnostic: every wait inside a kernel is bounded; a wait that runs out sets a bit of a
 * per-device word instead of hanging (bit 0: a barrier of the bulk-copy ring; bit 2: a
 * row slot of the one-block-per-SM forward).  This reads and clears that word for the
 * current device (*out = 0: no wait ran out).  Synchronises with the device.  No
 * counterpart in the reference.
 */
int k1_ring_status(unsigned* out);

/*
 * Device scratch needed by k1_fused_logprob_entropy_v1 and k1_vocab_shard_partials
 * for the cross-CTA combine of rows that are split between thread blocks.  The
 * workspace must be zero-filled before its first use; every call leaves it
 * zero-filled again, so one buffer can be reused by consecutive calls on one stream.
 * Calls that may overlap on the GPU need separate workspaces.  device = CUDA ordinal.
 */
size_t k1_forward_workspace_bytes(int64_t n_rows, int64_t vocab, int dtype, int device);

/*
 * Forward (production path).  Replaces fused_logprob_entropy_v1
 * (reference csrc/fused_logprob.cu:355-403, bound at csrc/bindings.cpp:21-23).
 *   logits   : rows x vocab elements of `dtype`, layout as described above
 *   targets  : n_rows int64, contiguous
 *   logprob, entropy, lse : n_rows fp32 each, contiguous (written)
 * One streaming read of the logits; every thread block gets an equal share of the
 * flattened row x vocab range, so few rows (split-vocab) and many rows use the same
 * kernel.
 */
int k1_fused_logprob_entropy_v1(const void* logits, int dtype, int64_t n_rows, int64_t vocab,
                                int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                                const int64_t* targets, float* logprob, float* entropy,
                                float* lse, void* workspace, size_t workspace_bytes,
                                void* stream);

/*
 * Forward that allocates nothing and takes no workspace: the same kernel and results as
 * k1_fused_logprob_entropy_v1, with its split-row scratch in a 512 KiB array that the
 * library defines in device memory (held on every GPU that loads the library until the
 * process exits).  For callers that cannot call cudaMalloc or hand out device memory of
 * their own -- e.g. a plugin inside a host framework whose memory pool is the only
 * allocator, or latency-critical code that must avoid cudaMalloc's implicit device
 * synchronisation.  Fails with K1_ERR_WORKSPACE if a device needs more scratch than the
 * array holds (it needs 2 x 24 + 4 bytes for each of 32 work owners per SM, about 241 KiB on
 * 148 SMs).
 * The first call on a device looks up the array's device address with that device
 * current; make that first call before any stream capture.  Each call clears the part
 * of the array that must start at zero.  All calls on a device share the array: calls
 * that may overlap on the GPU (different streams, concurrent host threads) race and must
 * be serialised by the caller.  The looked-up address is kept for the life of the
 * process: after cudaDeviceReset (or any reset of the device's primary context) the array
 * is reloaded at a new address, so calls after a reset are not supported.
 * No counterpart in the reference.
 */
int k1_fused_logprob_entropy_v1_noalloc(const void* logits, int dtype, int64_t n_rows,
                                        int64_t vocab, int64_t inner_rows, int64_t inner_stride,
                                        int64_t outer_stride, const int64_t* targets,
                                        float* logprob, float* entropy, float* lse, void* stream);

/*
 * Forward, one thread per row, fp64 accumulation.  A simple correctness anchor,
 * never fast.  Replaces fused_logprob_entropy_naive
 * (reference csrc/fused_logprob.cu:405-458, bound at csrc/bindings.cpp:18-20).
 */
int k1_fused_logprob_entropy_naive(const void* logits, int dtype, int64_t n_rows, int64_t vocab,
                                   int64_t inner_rows, int64_t inner_stride,
                                   int64_t outer_stride, const int64_t* targets,
                                   float* logprob, float* entropy, float* lse, void* stream);

/*
 * Backward.  Replaces fused_logprob_entropy_v1_backward
 * (reference csrc/fused_logprob.cu:284-346, bound at csrc/bindings.cpp:24-26):
 *   d_logits[r, v] = p (g_lse - g_logp - g_ent (x - lse + H)) + [v == t] g_logp,
 *   p = exp(x - lse), using the forward's saved lse and entropy (fp32, n_rows each).
 * g_logp / g_ent / g_lse may be NULL, meaning all-zero (the reference substitutes
 * zero tensors in Python, python/kernel_opt/ops.py:71-76).
 * d_logits has the dtype of logits and its own two-level row layout
 * (d_inner_stride, d_outer_stride; same inner_rows); d_logits == logits with the same
 * layout computes the gradient in place.
 */
int k1_fused_logprob_entropy_v1_backward(
    const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t inner_rows,
    int64_t inner_stride, int64_t outer_stride, const int64_t* targets, const float* lse,
    const float* entropy, const float* g_logp, const float* g_ent, const float* g_lse,
    void* d_logits, int64_t d_inner_stride, int64_t d_outer_stride, void* stream);

/*
 * Forward and backward with the logits scaled on the fly (the GRPO sampling temperature),
 * for the reference trainer's `logits.div_(self.temperature)` followed by K1 on the
 * completion window (reference python/kernel_opt/trainer.py:101-127).  Every logit x is read
 * as y = dtype(x * scale): the fp32 product rounded to nearest-even in the logits' type, which
 * is the tensor torch's in-place division leaves behind (torch divides a CUDA tensor by a
 * Python scalar T as a multiplication by the reciprocal taken in double and rounded to
 * fp32, so pass scale = (float)(1.0 / T); 1.0f / (float)T differs in the last bit for
 * some T, e.g. 0.85).  The forward
 * results are those of k1_fused_logprob_entropy_v1 on y, bit for bit; the backward writes the
 * gradient with respect to x, d_logits = dtype(dtype(dL/dy) * scale): K1's backward on y
 * followed by the division's own backward, again bit for bit.  The division pass, its
 * backward pass and the temporary that holds y are gone.  scale must be positive and finite;
 * scale == 1 runs the unscaled kernels.  All other arguments as for
 * k1_fused_logprob_entropy_v1 / _v1_backward (d_logits may alias logits: in place).
 * No single counterpart in the reference.
 */
int k1_fused_logprob_entropy_scaled(const void* logits, int dtype, int64_t n_rows,
                                    int64_t vocab, int64_t inner_rows, int64_t inner_stride,
                                    int64_t outer_stride, float scale, const int64_t* targets,
                                    float* logprob, float* entropy, float* lse, void* workspace,
                                    size_t workspace_bytes, void* stream);

int k1_fused_logprob_entropy_scaled_backward(
    const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t inner_rows,
    int64_t inner_stride, int64_t outer_stride, float scale, const int64_t* targets,
    const float* lse, const float* entropy, const float* g_logp, const float* g_ent,
    const float* g_lse, void* d_logits, int64_t d_inner_stride, int64_t d_outer_stride,
    void* stream);

/*
 * Vocab-parallel forward, step 1 of 3: per-row partial state of this rank's vocabulary
 * shard, columns [vocab_offset, vocab_offset + shard_vocab) of the full vocabulary.
 * `targets` hold global column ids.  partials: n_rows k1_partial (written).
 * No counterpart in the reference (multi-GPU was out of its scope).
 */
int k1_vocab_shard_partials(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab,
                            int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                            int64_t vocab_offset, const int64_t* targets,
                            k1_partial* partials, void* workspace, size_t workspace_bytes,
                            void* stream);

/*
 * Vocab-parallel forward, step 3 of 3 (step 2 is one all-gather of the partials):
 * gathered = n_shards x n_rows k1_partial (shard-major) -> logprob, entropy, lse.
 */
int k1_vocab_combine(const k1_partial* gathered, int n_shards, int64_t n_rows,
                     float* logprob, float* entropy, float* lse, void* stream);

/*
 * Vocab-parallel backward: the backward above restricted to this rank's shard, with
 * the global lse / entropy of the combined forward.  The one-hot term is applied only
 * where the global target falls inside [vocab_offset, vocab_offset + shard_vocab).
 */
int k1_vocab_shard_backward(
    const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab, int64_t inner_rows,
    int64_t inner_stride, int64_t outer_stride, int64_t vocab_offset, const int64_t* targets,
    const float* lse, const float* entropy, const float* g_logp, const float* g_ent,
    const float* g_lse, void* d_logits, int64_t d_inner_stride, int64_t d_outer_stride,
    void* stream);

/*
 * The same with the temperature folded in (the shard's logits read as dtype(x * scale),
 * as k1_fused_logprob_entropy_scaled_backward): the backward of a vocab-parallel LM head
 * that kept its logits shard.  d_logits may alias logits (in place).  No counterpart in
 * the reference.
 */
int k1_vocab_shard_scaled_backward(
    const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab, int64_t inner_rows,
    int64_t inner_stride, int64_t outer_stride, int64_t vocab_offset, float scale,
    const int64_t* targets, const float* lse, const float* entropy, const float* g_logp,
    const float* g_ent, const float* g_lse, void* d_logits, int64_t d_inner_stride,
    int64_t d_outer_stride, void* stream);

/*
 * LM head fused with K1 on the tensor cores (tcgen05).  The reference names this as its
 * follow-up and leaves it unbuilt (README.md:135-136, docs/FINAL_REPORT.md:490-494); the
 * unfused sequence it replaces is the model's LM head GEMM, then the trainer's
 * `logits.div_(temperature)` and K1 (python/kernel_opt/trainer.py:96-127).
 *   hidden : n_rows x hidden_dim bf16, row-major (rows hidden_dim elements apart)
 *   weight : vocab x hidden_dim bf16, row-major (the LM head's [V, H] weight)
 *   logits : z = bf16(hidden weight^T) (fp32 accumulation), read by K1 as
 *            y = bf16(z * scale), scale = 1/temperature (1 = no temperature)
 * hidden_dim must be a multiple of 8 and both matrices 16-byte aligned.
 *
 * Workspace bytes k1_lm_head_forward needs (per-row partials of the vocabulary runs);
 * 0 for invalid arguments.
 */
size_t k1_lm_head_workspace_bytes(int64_t n_rows, int64_t hidden_dim, int64_t vocab, int device);

/*
 * Forward: logprob, entropy, lse (n_rows fp32 each) of K1 on the logits above, computed
 * tile by tile in the GEMM's epilogue.  logits_out = NULL: the logits never reach memory;
 * otherwise z is also written to logits_out (rows logits_stride >= vocab elements apart),
 * for a backward that keeps them.  targets: n_rows int64 (outside [0, vocab): logprob =
 * -lse, as in K1).
 */
int k1_lm_head_forward(const void* hidden, const void* weight, int64_t n_rows, int64_t hidden_dim,
                       int64_t vocab, float scale, const int64_t* targets, float* logprob,
                       float* entropy, float* lse, void* logits_out, int64_t logits_stride,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward to the logits: recomputes each logits tile on the tensor cores and writes
 * d_logits = dtype(dtype(dL/dy) * scale), exactly what
 * k1_fused_logprob_entropy_scaled_backward writes for the logits z (bf16, rows d_stride >=
 * vocab elements apart), from the forward's lse and entropy and the upstream gradients
 * (NULL = zero).  The caller then forms dL/dhidden = d_logits weight and
 * dL/dweight = d_logits^T hidden.
 */
int k1_lm_head_backward(const void* hidden, const void* weight, int64_t n_rows, int64_t hidden_dim,
                        int64_t vocab, float scale, const int64_t* targets, const float* lse,
                        const float* entropy, const float* g_logp, const float* g_ent,
                        const float* g_lse, void* d_logits, int64_t d_stride, void* stream);

/*
 * The LM head split over the vocabulary (tensor-parallel head: this rank holds rows
 * [vocab_offset, vocab_offset + shard_vocab) of the [V, H] weight, weight_shard pointing at
 * the first).  No counterpart in the reference (single GPU, LM head unbuilt); the rows'
 * combine is the vocab-parallel one above.
 *
 * Forward, step 1 of 3: each row's k1_partial over this shard's logits, computed in the
 * tensor-core kernel's epilogue; `targets` hold global token ids.  logits_out = NULL: the
 * logits never reach memory; otherwise the shard's z is also written (rows logits_stride
 * >= shard_vocab elements apart) for a backward that keeps it
 * (k1_vocab_shard_scaled_backward).  Workspace: k1_lm_head_workspace_bytes(n_rows,
 * hidden_dim, shard_vocab, dev).
 * Steps 2 and 3 are the all-gather of the partials and k1_vocab_combine.
 */
int k1_lm_head_shard_partials(const void* hidden, const void* weight_shard, int64_t n_rows,
                              int64_t hidden_dim, int64_t shard_vocab, int64_t vocab_offset,
                              float scale, const int64_t* targets, k1_partial* partials,
                              void* logits_out, int64_t logits_stride, void* workspace,
                              size_t workspace_bytes, void* stream);

/*
 * Backward to this shard's logits: k1_lm_head_backward on the shard, with the global lse /
 * entropy of the combined forward; the one-hot term only where the target lies in the
 * shard.  d_logits: n_rows x shard_vocab bf16 (rows d_stride >= shard_vocab elements apart).
 * The caller forms this shard's dL/dweight = d_logits^T hidden and its part of
 * dL/dhidden = d_logits weight_shard (summed over the shards).
 */
int k1_lm_head_shard_backward(const void* hidden, const void* weight_shard, int64_t n_rows,
                              int64_t hidden_dim, int64_t shard_vocab, int64_t vocab_offset,
                              float scale, const int64_t* targets, const float* lse,
                              const float* entropy, const float* g_logp, const float* g_ent,
                              const float* g_lse, void* d_logits, int64_t d_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* K1_LOGPROB_H */
