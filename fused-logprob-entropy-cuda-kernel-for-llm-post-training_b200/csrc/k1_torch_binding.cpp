// k1_torch_binding.cpp -- the `kernel_opt._C` torch extension.
//
// Mirrors the reference binding (csrc/bindings.cpp:3-26): the same three functions with
// the same out-parameter signatures and the same TORCH_CHECK messages as the reference
// host dispatch (csrc/fused_logprob.cu:284-458), so `RuntimeError`s read the same.  The
// work itself goes through the C ABI of libk1_b200.so (include/k1_logprob.h); this file
// only turns tensors into pointers, strides and the current CUDA stream.
//
// Deliberate relaxations of the reference's checks:
//  * logits need unit stride on the vocab axis only; leading dims must collapse to at
//    most two stride levels (e.g. logits[:, :-1, :] of a [B, L, V] tensor);
//  * backward upstream gradients may be None (treated as zero);
//  * d_logits may have any layout of the same kind (and may alias logits).
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <atomic>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "k1_logprob.h"

namespace {

struct Rows {
    int64_t n_rows = 0, vocab = 0, inner_rows = 1, inner_stride = 0, outer_stride = 0;
};

// Collapse the leading dims of x[..., V] (stride(-1) == 1) into the two-level layout of
// the C ABI.  Returns false when the leading dims need more than two stride levels.
bool rows_of(const at::Tensor& x, Rows& L) {
    const int64_t nd = x.dim();
    L.vocab = x.size(nd - 1);
    std::vector<std::pair<int64_t, int64_t>> dims;  // (size, stride) with size > 1
    int64_t n = 1;
    for (int64_t d = 0; d < nd - 1; ++d) {
        n *= x.size(d);
        if (x.size(d) != 1) dims.emplace_back(x.size(d), x.stride(d));
    }
    L.n_rows = n;
    // merge dims that are contiguous with respect to each other
    std::vector<std::pair<int64_t, int64_t>> m;
    for (auto& d : dims) {
        if (!m.empty() && m.back().second == d.first * d.second) {
            m.back().first *= d.first;
            m.back().second = d.second;
        } else {
            m.push_back(d);
        }
    }
    if (m.empty()) {
        L.inner_rows = 1;
        L.inner_stride = L.vocab;
        L.outer_stride = L.vocab;
        return true;
    }
    if (m.size() == 1) {
        L.inner_rows = m[0].first;
        L.inner_stride = m[0].second;
        L.outer_stride = m[0].first * m[0].second;
        return true;
    }
    if (m.size() == 2) {
        L.inner_rows = m[1].first;
        L.inner_stride = m[1].second;
        L.outer_stride = m[0].second;
        return true;
    }
    return false;
}

int dtype_code(const at::Tensor& x) {
    if (x.scalar_type() == at::kBFloat16) return K1_DTYPE_BF16;
    if (x.scalar_type() == at::kHalf) return K1_DTYPE_F16;
    if (x.scalar_type() == at::kFloat) return K1_DTYPE_F32;
    return -1;
}

void check_rc(int rc) {
    TORCH_CHECK(rc == K1_OK, k1_last_error());
}

// Opt-in check of the kernels' bounded waits (K1_CHECK_WAITS=1 in the environment, or
// _C.set_check_waits(True)).  A wait inside a kernel that runs out sets a device word and
// leaves NaN in the outputs it could not finish; with the check on, every compute call
// then synchronises its stream, reads and clears that word and raises.  Off by default
// (it synchronises); skipped while the current stream is being captured into a graph.
std::atomic<bool>& check_waits_flag() {
    static std::atomic<bool> flag{[] {
        const char* e = std::getenv("K1_CHECK_WAITS");
        return e != nullptr && e[0] != '\0' && e[0] != '0';
    }()};
    return flag;
}

void check_launch(int rc) {
    check_rc(rc);
    if (!check_waits_flag().load(std::memory_order_relaxed)) return;
    cudaStream_t s = at::cuda::getCurrentCUDAStream().stream();
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return;
    const cudaError_t e = cudaStreamSynchronize(s);
    TORCH_CHECK(e == cudaSuccess, "k1: ", cudaGetErrorString(e));
    unsigned v = 0;
    check_rc(k1_ring_status(&v));
    TORCH_CHECK(v == 0, "k1: a bounded wait inside a K1 kernel ran out (status ", v,
                "); the outputs it could not finish hold NaN");
}

Rows logits_rows(const at::Tensor& logits) {
    TORCH_CHECK(logits.dim() >= 1, "logits must have a vocab dimension");
    TORCH_CHECK(logits.size(-1) == 0 || logits.stride(-1) == 1 || logits.size(-1) == 1,
                "logits must be contiguous along the vocab dimension");
    Rows L;
    TORCH_CHECK(rows_of(logits, L),
                "logits must be contiguous, or a view whose leading dims collapse to two "
                "strided levels with unit vocab stride");
    return L;
}

// Persistent zero-initialised forward workspace, one per (device, stream); the kernels
// leave it zeroed after every call.  Never freed (kept alive until process exit).
void* forward_workspace(const at::Tensor& like, size_t* bytes) {
    static std::mutex mu;
    static auto* cache = new std::map<std::pair<int, cudaStream_t>, at::Tensor>();
    const int dev = like.get_device();
    cudaStream_t s = at::cuda::getCurrentCUDAStream(dev).stream();
    const size_t need = k1_forward_workspace_bytes(0, 0, 0, dev);
    TORCH_CHECK(need > 0, "k1: could not size the forward workspace: ", k1_last_error());
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_pair(dev, s);
    auto it = cache->find(key);
    if (it == cache->end() || (size_t)it->second.numel() < need) {
        at::Tensor ws = at::zeros({(int64_t)need}, like.options().dtype(at::kByte));
        it = cache->insert_or_assign(key, ws).first;
    }
    *bytes = (size_t)it->second.numel();
    return it->second.data_ptr();
}

void check_fwd_common(const at::Tensor& logits, const at::Tensor& targets,
                      const at::Tensor& logprob, const at::Tensor& entropy,
                      const at::Tensor& lse_out, int64_t n_rows) {
    TORCH_CHECK(logits.is_cuda(), "logits must be CUDA");
    TORCH_CHECK(targets.is_cuda(), "targets must be CUDA");
    TORCH_CHECK(targets.scalar_type() == at::kLong, "targets must be int64");
    TORCH_CHECK(targets.is_contiguous(), "targets must be contiguous");
    TORCH_CHECK(logprob.scalar_type() == at::kFloat && entropy.scalar_type() == at::kFloat &&
                    lse_out.scalar_type() == at::kFloat,
                "outputs must be float32");
    TORCH_CHECK(logprob.is_contiguous() && entropy.is_contiguous() && lse_out.is_contiguous(),
                "outputs must be contiguous");
    TORCH_CHECK(logprob.is_cuda() && entropy.is_cuda() && lse_out.is_cuda(),
                "outputs must be CUDA");
    TORCH_CHECK(targets.get_device() == logits.get_device() &&
                    logprob.get_device() == logits.get_device() &&
                    entropy.get_device() == logits.get_device() &&
                    lse_out.get_device() == logits.get_device(),
                "all tensors must be on the same device");
    TORCH_CHECK(targets.numel() == n_rows, "targets numel must match leading dims of logits");
    TORCH_CHECK(logprob.numel() == n_rows && entropy.numel() == n_rows && lse_out.numel() == n_rows,
                "output tensor numels must equal leading-dim count");
}

// _C.fused_logprob_entropy_v1 (reference csrc/fused_logprob.cu:355-403)
void fused_logprob_entropy_v1(at::Tensor logits, at::Tensor targets, at::Tensor logprob,
                              at::Tensor entropy, at::Tensor lse_out) {
    const int dt = dtype_code(logits);
    TORCH_CHECK(dt >= 0, "logits dtype must be bf16, fp16, or fp32");
    Rows L = logits_rows(logits);
    check_fwd_common(logits, targets, logprob, entropy, lse_out, L.n_rows);
    if (L.n_rows == 0) return;
    c10::cuda::CUDAGuard guard(logits.device());
    size_t ws_bytes = 0;
    void* ws = forward_workspace(logits, &ws_bytes);
    check_launch(k1_fused_logprob_entropy_v1(
        logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows, L.inner_stride, L.outer_stride,
        targets.data_ptr<int64_t>(), logprob.data_ptr<float>(), entropy.data_ptr<float>(),
        lse_out.data_ptr<float>(), ws, ws_bytes, at::cuda::getCurrentCUDAStream().stream()));
}

// _C.fused_logprob_entropy_scaled: the forward on logits read as dtype(x * scale) (the
// GRPO temperature, scale = 1/T in fp32), in place of `logits.div_(T)` + K1 (reference
// python/kernel_opt/trainer.py:101-127).
void fused_logprob_entropy_scaled(at::Tensor logits, at::Tensor targets, at::Tensor logprob,
                                  at::Tensor entropy, at::Tensor lse_out, double scale) {
    const int dt = dtype_code(logits);
    TORCH_CHECK(dt >= 0, "logits dtype must be bf16, fp16, or fp32");
    Rows L = logits_rows(logits);
    check_fwd_common(logits, targets, logprob, entropy, lse_out, L.n_rows);
    if (L.n_rows == 0) return;
    c10::cuda::CUDAGuard guard(logits.device());
    size_t ws_bytes = 0;
    void* ws = forward_workspace(logits, &ws_bytes);
    check_launch(k1_fused_logprob_entropy_scaled(
        logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows, L.inner_stride, L.outer_stride,
        (float)scale, targets.data_ptr<int64_t>(), logprob.data_ptr<float>(),
        entropy.data_ptr<float>(), lse_out.data_ptr<float>(), ws, ws_bytes,
        at::cuda::getCurrentCUDAStream().stream()));
}

// _C.fused_logprob_entropy_naive (reference csrc/fused_logprob.cu:405-458)
void fused_logprob_entropy_naive(at::Tensor logits, at::Tensor targets, at::Tensor logprob,
                                 at::Tensor entropy, at::Tensor lse_out) {
    const int dt = dtype_code(logits);
    TORCH_CHECK(dt >= 0, "logits dtype must be bf16, fp16, or fp32");
    Rows L = logits_rows(logits);
    check_fwd_common(logits, targets, logprob, entropy, lse_out, L.n_rows);
    if (L.n_rows == 0) return;
    c10::cuda::CUDAGuard guard(logits.device());
    check_launch(k1_fused_logprob_entropy_naive(
        logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows, L.inner_stride, L.outer_stride,
        targets.data_ptr<int64_t>(), logprob.data_ptr<float>(), entropy.data_ptr<float>(),
        lse_out.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()));
}

const float* opt_grad(const c10::optional<at::Tensor>& g, int64_t n_rows, const at::Tensor& like) {
    if (!g.has_value() || !g->defined()) return nullptr;
    TORCH_CHECK(g->scalar_type() == at::kFloat, "upstream gradients must be fp32");
    TORCH_CHECK(g->is_contiguous(), "upstream gradients must be contiguous");
    TORCH_CHECK(g->is_cuda() && g->get_device() == like.get_device(),
                "upstream gradients must be on the logits' device");
    TORCH_CHECK(g->numel() == n_rows, "leading-dim count mismatch");
    return g->data_ptr<float>();
}

void backward_common(const char* which, at::Tensor logits, at::Tensor targets, int64_t vocab_offset,
                     at::Tensor lse, at::Tensor entropy, c10::optional<at::Tensor> g_logp,
                     c10::optional<at::Tensor> g_ent, c10::optional<at::Tensor> g_lse,
                     at::Tensor d_logits, double scale = 1.0) {
    TORCH_CHECK(logits.is_cuda(), "logits must be contiguous CUDA");
    TORCH_CHECK(targets.scalar_type() == at::kLong, "targets must be int64");
    TORCH_CHECK(targets.is_contiguous() && targets.is_cuda(), "targets must be contiguous CUDA");
    TORCH_CHECK(lse.scalar_type() == at::kFloat && entropy.scalar_type() == at::kFloat,
                "saved lse / entropy must be fp32");
    TORCH_CHECK(lse.is_contiguous() && entropy.is_contiguous(), "saved lse / entropy must be contiguous");
    const int dt = dtype_code(logits);
    TORCH_CHECK(dt >= 0, "logits dtype must be bf16, fp16, or fp32");
    TORCH_CHECK(d_logits.scalar_type() == logits.scalar_type() && d_logits.sizes() == logits.sizes(),
                "d_logits must match logits dtype/shape");
    TORCH_CHECK(d_logits.is_cuda() && d_logits.get_device() == logits.get_device(),
                "d_logits must be on the logits' device");
    Rows L = logits_rows(logits);
    TORCH_CHECK(targets.numel() == L.n_rows && lse.numel() == L.n_rows && entropy.numel() == L.n_rows,
                "leading-dim count mismatch");
    const float* gl = opt_grad(g_logp, L.n_rows, logits);
    const float* ge = opt_grad(g_ent, L.n_rows, logits);
    const float* gs = opt_grad(g_lse, L.n_rows, logits);
    if (L.n_rows == 0) return;
    // logits and d_logits share one row grouping (inner_rows): try the grouping of each
    // tensor, view both as [n_rows / k, k, V] (no copy) and read their row strides.
    TORCH_CHECK(d_logits.size(-1) == 1 || d_logits.stride(-1) == 1,
                "d_logits must be contiguous along the vocab dimension");
    Rows D = logits_rows(d_logits);
    bool found = false;
    for (int64_t k : {L.inner_rows, D.inner_rows}) {
        if (k < 1 || L.n_rows % k != 0) continue;
        try {
            at::Tensor lv = logits.view({L.n_rows / k, k, L.vocab});
            at::Tensor dv = d_logits.view({L.n_rows / k, k, L.vocab});
            L.inner_rows = D.inner_rows = k;
            L.inner_stride = lv.stride(1);
            L.outer_stride = lv.stride(0);
            D.inner_stride = dv.stride(1);
            D.outer_stride = dv.stride(0);
            found = true;
            break;
        } catch (const c10::Error&) {
        }
    }
    TORCH_CHECK(found, "d_logits layout cannot be addressed with the logits' row grouping");
    c10::cuda::CUDAGuard guard(logits.device());
    cudaStream_t s = at::cuda::getCurrentCUDAStream().stream();
    int rc;
    if (which[0] == 'v' && scale != 1.0) {
        rc = k1_vocab_shard_scaled_backward(
            logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows, L.inner_stride, L.outer_stride,
            vocab_offset, (float)scale, targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
            entropy.data_ptr<float>(), gl, ge, gs, d_logits.data_ptr(), D.inner_stride,
            D.outer_stride, s);
    } else if (which[0] == 'v') {
        rc = k1_vocab_shard_backward(logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows,
                                     L.inner_stride, L.outer_stride, vocab_offset,
                                     targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
                                     entropy.data_ptr<float>(), gl, ge, gs, d_logits.data_ptr(),
                                     D.inner_stride, D.outer_stride, s);
    } else if (which[0] == 's') {
        rc = k1_fused_logprob_entropy_scaled_backward(
            logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows, L.inner_stride, L.outer_stride,
            (float)scale, targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
            entropy.data_ptr<float>(), gl, ge, gs, d_logits.data_ptr(), D.inner_stride,
            D.outer_stride, s);
    } else {
        rc = k1_fused_logprob_entropy_v1_backward(
            logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows, L.inner_stride, L.outer_stride,
            targets.data_ptr<int64_t>(), lse.data_ptr<float>(), entropy.data_ptr<float>(), gl, ge,
            gs, d_logits.data_ptr(), D.inner_stride, D.outer_stride, s);
    }
    check_launch(rc);
}

// _C.fused_logprob_entropy_v1_backward (reference csrc/fused_logprob.cu:284-346)
void fused_logprob_entropy_v1_backward(at::Tensor logits, at::Tensor targets, at::Tensor lse,
                                       at::Tensor entropy, c10::optional<at::Tensor> g_logp,
                                       c10::optional<at::Tensor> g_ent,
                                       c10::optional<at::Tensor> g_lse, at::Tensor d_logits) {
    backward_common("b", logits, targets, 0, lse, entropy, g_logp, g_ent, g_lse, d_logits);
}

// _C.fused_logprob_entropy_scaled_backward: gradient w.r.t. the unscaled logits x,
// dtype(dtype(dL/dy) * scale) with y = dtype(x * scale).
void fused_logprob_entropy_scaled_backward(at::Tensor logits, at::Tensor targets, at::Tensor lse,
                                           at::Tensor entropy, c10::optional<at::Tensor> g_logp,
                                           c10::optional<at::Tensor> g_ent,
                                           c10::optional<at::Tensor> g_lse, at::Tensor d_logits,
                                           double scale) {
    backward_common("s", logits, targets, 0, lse, entropy, g_logp, g_ent, g_lse, d_logits, scale);
}

// Vocab-parallel step 1: partials [n_rows, 4] float64 (one k1_partial per row).
void vocab_shard_partials(at::Tensor logits, at::Tensor targets, int64_t vocab_offset,
                          at::Tensor partials) {
    const int dt = dtype_code(logits);
    TORCH_CHECK(dt >= 0, "logits dtype must be bf16, fp16, or fp32");
    TORCH_CHECK(logits.is_cuda() && targets.is_cuda() && partials.is_cuda(),
                "logits, targets and partials must be CUDA");
    TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(),
                "targets must be contiguous int64");
    Rows L = logits_rows(logits);
    TORCH_CHECK(targets.numel() == L.n_rows, "targets numel must match leading dims of logits");
    TORCH_CHECK(partials.scalar_type() == at::kDouble && partials.is_contiguous() &&
                    partials.numel() == 4 * L.n_rows,
                "partials must be a contiguous float64 tensor of n_rows x 4");
    if (L.n_rows == 0) return;
    c10::cuda::CUDAGuard guard(logits.device());
    size_t ws_bytes = 0;
    void* ws = forward_workspace(logits, &ws_bytes);
    check_launch(k1_vocab_shard_partials(logits.data_ptr(), dt, L.n_rows, L.vocab, L.inner_rows,
                                     L.inner_stride, L.outer_stride, vocab_offset,
                                     targets.data_ptr<int64_t>(),
                                     reinterpret_cast<k1_partial*>(partials.data_ptr()), ws,
                                     ws_bytes, at::cuda::getCurrentCUDAStream().stream()));
}

// Vocab-parallel step 3: gathered [n_shards, n_rows, 4] float64 -> outputs.
void vocab_combine(at::Tensor gathered, int64_t n_shards, at::Tensor logprob, at::Tensor entropy,
                   at::Tensor lse_out) {
    TORCH_CHECK(gathered.is_cuda() && gathered.scalar_type() == at::kDouble &&
                    gathered.is_contiguous(),
                "gathered partials must be a contiguous CUDA float64 tensor");
    TORCH_CHECK(n_shards >= 1, "n_shards must be >= 1");
    const int64_t n_rows = logprob.numel();
    TORCH_CHECK(gathered.numel() == 4 * n_shards * n_rows,
                "gathered partials must hold n_shards x n_rows x 4 values");
    TORCH_CHECK(logprob.scalar_type() == at::kFloat && entropy.scalar_type() == at::kFloat &&
                    lse_out.scalar_type() == at::kFloat,
                "outputs must be float32");
    TORCH_CHECK(entropy.numel() == n_rows && lse_out.numel() == n_rows,
                "output tensor numels must equal leading-dim count");
    TORCH_CHECK(logprob.is_contiguous() && entropy.is_contiguous() && lse_out.is_contiguous(),
                "outputs must be contiguous");
    if (n_rows == 0) return;
    c10::cuda::CUDAGuard guard(gathered.device());
    check_launch(k1_vocab_combine(reinterpret_cast<const k1_partial*>(gathered.data_ptr()),
                              (int)n_shards, n_rows, logprob.data_ptr<float>(),
                              entropy.data_ptr<float>(), lse_out.data_ptr<float>(),
                              at::cuda::getCurrentCUDAStream().stream()));
}

// Vocab-parallel backward of one shard.
void vocab_shard_backward(at::Tensor logits, at::Tensor targets, int64_t vocab_offset,
                          at::Tensor lse, at::Tensor entropy, c10::optional<at::Tensor> g_logp,
                          c10::optional<at::Tensor> g_ent, c10::optional<at::Tensor> g_lse,
                          at::Tensor d_logits, double scale) {
    // scale != 1: the shard's logits are read as dtype(x * scale) (temperature folded in)
    backward_common("v", logits, targets, vocab_offset, lse, entropy, g_logp, g_ent, g_lse,
                    d_logits, scale);
}

// LM head fused with K1 on the tensor cores (bf16 hidden [N, H] and weight [V, H]).
void check_lm_head(const at::Tensor& hidden, const at::Tensor& weight, const at::Tensor& targets) {
    TORCH_CHECK(hidden.is_cuda() && weight.is_cuda() && targets.is_cuda(),
                "hidden, weight and targets must be CUDA");
    TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && weight.scalar_type() == at::kBFloat16,
                "the tensor-core LM head takes bf16 hidden and weight");
    TORCH_CHECK(hidden.dim() == 2 && weight.dim() == 2 && hidden.size(1) == weight.size(1),
                "hidden [N, H] and weight [V, H] expected");
    TORCH_CHECK(hidden.is_contiguous() && weight.is_contiguous(), "hidden and weight must be contiguous");
    TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous() &&
                    targets.numel() == hidden.size(0),
                "targets must be contiguous int64 with one entry per hidden row");
    TORCH_CHECK(hidden.get_device() == weight.get_device() && hidden.get_device() == targets.get_device(),
                "hidden, weight and targets must be on one device");
}

void lm_head_forward(at::Tensor hidden, at::Tensor weight, at::Tensor targets, at::Tensor logprob,
                     at::Tensor entropy, at::Tensor lse_out, double scale,
                     c10::optional<at::Tensor> logits_out) {
    check_lm_head(hidden, weight, targets);
    const int64_t N = hidden.size(0), H = hidden.size(1), V = weight.size(0);
    for (const at::Tensor* o : {&logprob, &entropy, &lse_out})
        TORCH_CHECK(o->scalar_type() == at::kFloat && o->is_contiguous() && o->numel() == N,
                    "outputs must be contiguous fp32 with one entry per row");
    void* zp = nullptr;
    int64_t zs = V;
    if (logits_out.has_value() && logits_out->defined()) {
        const at::Tensor& z = *logits_out;
        TORCH_CHECK(z.scalar_type() == at::kBFloat16 && z.dim() == 2 && z.size(0) == N &&
                        z.size(1) == V && z.stride(1) == 1,
                    "logits_out must be bf16 [N, V] with unit stride along V");
        zp = z.data_ptr();
        zs = z.stride(0);
    }
    if (N == 0) return;
    c10::cuda::CUDAGuard guard(hidden.device());
    const size_t ws_bytes = k1_lm_head_workspace_bytes(N, H, V, hidden.get_device());
    TORCH_CHECK(ws_bytes > 0, "k1: could not size the LM head workspace: ", k1_last_error());
    at::Tensor ws = at::empty({(int64_t)ws_bytes}, hidden.options().dtype(at::kByte));
    check_launch(k1_lm_head_forward(hidden.data_ptr(), weight.data_ptr(), N, H, V, (float)scale,
                                    targets.data_ptr<int64_t>(), logprob.data_ptr<float>(),
                                    entropy.data_ptr<float>(), lse_out.data_ptr<float>(), zp, zs,
                                    ws.data_ptr(), ws_bytes,
                                    at::cuda::getCurrentCUDAStream().stream()));
}

void lm_head_backward(at::Tensor hidden, at::Tensor weight, at::Tensor targets, at::Tensor lse,
                      at::Tensor entropy, c10::optional<at::Tensor> g_logp,
                      c10::optional<at::Tensor> g_ent, c10::optional<at::Tensor> g_lse,
                      at::Tensor d_logits, double scale) {
    check_lm_head(hidden, weight, targets);
    const int64_t N = hidden.size(0), H = hidden.size(1), V = weight.size(0);
    TORCH_CHECK(lse.scalar_type() == at::kFloat && entropy.scalar_type() == at::kFloat &&
                    lse.is_contiguous() && entropy.is_contiguous() && lse.numel() == N &&
                    entropy.numel() == N,
                "saved lse / entropy must be contiguous fp32 with one entry per row");
    TORCH_CHECK(d_logits.scalar_type() == at::kBFloat16 && d_logits.dim() == 2 &&
                    d_logits.size(0) == N && d_logits.size(1) == V && d_logits.stride(1) == 1,
                "d_logits must be bf16 [N, V] with unit stride along V");
    const float* gl = opt_grad(g_logp, N, hidden);
    const float* ge = opt_grad(g_ent, N, hidden);
    const float* gs = opt_grad(g_lse, N, hidden);
    if (N == 0) return;
    c10::cuda::CUDAGuard guard(hidden.device());
    check_launch(k1_lm_head_backward(hidden.data_ptr(), weight.data_ptr(), N, H, V, (float)scale,
                                     targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
                                     entropy.data_ptr<float>(), gl, ge, gs, d_logits.data_ptr(),
                                     d_logits.stride(0), at::cuda::getCurrentCUDAStream().stream()));
}

// The LM head over a vocabulary shard (rows [vocab_offset, vocab_offset + weight.size(0)) of
// the full weight): per-row k1_partial of the shard, for the all-gather and vocab_combine.
void lm_head_shard_partials(at::Tensor hidden, at::Tensor weight, at::Tensor targets,
                            int64_t vocab_offset, at::Tensor partials, double scale,
                            c10::optional<at::Tensor> logits_out) {
    check_lm_head(hidden, weight, targets);
    const int64_t N = hidden.size(0), H = hidden.size(1), V = weight.size(0);
    TORCH_CHECK(partials.is_cuda() && partials.scalar_type() == at::kDouble &&
                    partials.is_contiguous() && partials.numel() == 4 * N,
                "partials must be a contiguous CUDA float64 tensor of n_rows x 4");
    void* zp = nullptr;
    int64_t zs = V;
    if (logits_out.has_value() && logits_out->defined()) {
        const at::Tensor& z = *logits_out;
        TORCH_CHECK(z.scalar_type() == at::kBFloat16 && z.dim() == 2 && z.size(0) == N &&
                        z.size(1) == V && z.stride(1) == 1,
                    "logits_out must be bf16 [N, V_shard] with unit stride along V");
        zp = z.data_ptr();
        zs = z.stride(0);
    }
    if (N == 0) return;
    c10::cuda::CUDAGuard guard(hidden.device());
    const size_t ws_bytes = k1_lm_head_workspace_bytes(N, H, V, hidden.get_device());
    TORCH_CHECK(ws_bytes > 0, "k1: could not size the LM head workspace: ", k1_last_error());
    at::Tensor ws = at::empty({(int64_t)ws_bytes}, hidden.options().dtype(at::kByte));
    check_launch(k1_lm_head_shard_partials(
        hidden.data_ptr(), weight.data_ptr(), N, H, V, vocab_offset, (float)scale,
        targets.data_ptr<int64_t>(), reinterpret_cast<k1_partial*>(partials.data_ptr()), zp, zs,
        ws.data_ptr(), ws_bytes, at::cuda::getCurrentCUDAStream().stream()));
}

void lm_head_shard_backward(at::Tensor hidden, at::Tensor weight, at::Tensor targets,
                            int64_t vocab_offset, at::Tensor lse, at::Tensor entropy,
                            c10::optional<at::Tensor> g_logp, c10::optional<at::Tensor> g_ent,
                            c10::optional<at::Tensor> g_lse, at::Tensor d_logits, double scale) {
    check_lm_head(hidden, weight, targets);
    const int64_t N = hidden.size(0), H = hidden.size(1), V = weight.size(0);
    TORCH_CHECK(lse.scalar_type() == at::kFloat && entropy.scalar_type() == at::kFloat &&
                    lse.is_contiguous() && entropy.is_contiguous() && lse.numel() == N &&
                    entropy.numel() == N,
                "saved lse / entropy must be contiguous fp32 with one entry per row");
    TORCH_CHECK(d_logits.scalar_type() == at::kBFloat16 && d_logits.dim() == 2 &&
                    d_logits.size(0) == N && d_logits.size(1) == V && d_logits.stride(1) == 1,
                "d_logits must be bf16 [N, V_shard] with unit stride along V");
    const float* gl = opt_grad(g_logp, N, hidden);
    const float* ge = opt_grad(g_ent, N, hidden);
    const float* gs = opt_grad(g_lse, N, hidden);
    if (N == 0) return;
    c10::cuda::CUDAGuard guard(hidden.device());
    check_launch(k1_lm_head_shard_backward(
        hidden.data_ptr(), weight.data_ptr(), N, H, V, vocab_offset, (float)scale,
        targets.data_ptr<int64_t>(), lse.data_ptr<float>(), entropy.data_ptr<float>(), gl, ge, gs,
        d_logits.data_ptr(), d_logits.stride(0), at::cuda::getCurrentCUDAStream().stream()));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("fused_logprob_entropy_naive", &fused_logprob_entropy_naive,
          "Forward, one thread per row in fp64 (correctness anchor).");
    m.def("fused_logprob_entropy_v1", &fused_logprob_entropy_v1,
          "Forward: one streaming pass, split evenly over all SMs.");
    m.def("fused_logprob_entropy_v1_backward", &fused_logprob_entropy_v1_backward,
          "Backward: streaming, recomputes softmax from the saved lse.", pybind11::arg("logits"),
          pybind11::arg("targets"), pybind11::arg("lse"), pybind11::arg("entropy"),
          pybind11::arg("g_logp"), pybind11::arg("g_ent"), pybind11::arg("g_lse"),
          pybind11::arg("d_logits"));
    m.def("fused_logprob_entropy_scaled", &fused_logprob_entropy_scaled,
          "Forward on logits read as dtype(x * scale) (temperature folded in).",
          pybind11::arg("logits"), pybind11::arg("targets"), pybind11::arg("logprob"),
          pybind11::arg("entropy"), pybind11::arg("lse_out"), pybind11::arg("scale"));
    m.def("fused_logprob_entropy_scaled_backward", &fused_logprob_entropy_scaled_backward,
          "Backward of the scaled forward, gradient w.r.t. the unscaled logits.",
          pybind11::arg("logits"), pybind11::arg("targets"), pybind11::arg("lse"),
          pybind11::arg("entropy"), pybind11::arg("g_logp"), pybind11::arg("g_ent"),
          pybind11::arg("g_lse"), pybind11::arg("d_logits"), pybind11::arg("scale"));
    m.def("vocab_shard_partials", &vocab_shard_partials,
          "Vocab-parallel: per-row partial state of a vocabulary shard.");
    m.def("vocab_combine", &vocab_combine, "Vocab-parallel: merge gathered shard partials.");
    m.def("vocab_shard_backward", &vocab_shard_backward,
          "Vocab-parallel: backward of a shard (scale != 1: logits read as dtype(x * scale)).",
          pybind11::arg("logits"), pybind11::arg("targets"), pybind11::arg("vocab_offset"),
          pybind11::arg("lse"), pybind11::arg("entropy"), pybind11::arg("g_logp"),
          pybind11::arg("g_ent"), pybind11::arg("g_lse"), pybind11::arg("d_logits"),
          pybind11::arg("scale") = 1.0);
    m.def("lm_head_forward", &lm_head_forward,
          "LM head fused with K1 on the tensor cores: per-row logprob / entropy / lse of "
          "bf16(hidden weight^T) read as bf16(z * scale); optionally also writes z.",
          pybind11::arg("hidden"), pybind11::arg("weight"), pybind11::arg("targets"),
          pybind11::arg("logprob"), pybind11::arg("entropy"), pybind11::arg("lse_out"),
          pybind11::arg("scale"), pybind11::arg("logits_out") = pybind11::none());
    m.def("lm_head_backward", &lm_head_backward,
          "Recomputes the LM head's logits on the tensor cores and writes K1's gradient "
          "w.r.t. them (the scaled backward's rounding).",
          pybind11::arg("hidden"), pybind11::arg("weight"), pybind11::arg("targets"),
          pybind11::arg("lse"), pybind11::arg("entropy"), pybind11::arg("g_logp"),
          pybind11::arg("g_ent"), pybind11::arg("g_lse"), pybind11::arg("d_logits"),
          pybind11::arg("scale"));
    m.def("lm_head_shard_partials", &lm_head_shard_partials,
          "Vocab-parallel LM head: per-row partial state of this rank's weight shard, from "
          "the tensor-core kernel's epilogue.",
          pybind11::arg("hidden"), pybind11::arg("weight"), pybind11::arg("targets"),
          pybind11::arg("vocab_offset"), pybind11::arg("partials"), pybind11::arg("scale"),
          pybind11::arg("logits_out") = pybind11::none());
    m.def("lm_head_shard_backward", &lm_head_shard_backward,
          "Vocab-parallel LM head: K1's gradient w.r.t. this shard's logits, recomputed on "
          "the tensor cores, from the combined lse / entropy.",
          pybind11::arg("hidden"), pybind11::arg("weight"), pybind11::arg("targets"),
          pybind11::arg("vocab_offset"), pybind11::arg("lse"), pybind11::arg("entropy"),
          pybind11::arg("g_logp"), pybind11::arg("g_ent"), pybind11::arg("g_lse"),
          pybind11::arg("d_logits"), pybind11::arg("scale"));
    m.def("abi_version", &k1_abi_version, "C ABI version of the loaded libk1_b200.so.");
    m.def(
        "ring_status",
        []() {
            unsigned v = 0;
            check_rc(k1_ring_status(&v));
            return v;
        },
        "Read and clear the bulk-copy ring's timeout word of the current device (0 = ok).");
    m.def(
        "set_check_waits", [](bool on) { check_waits_flag().store(on); },
        "Raise after any K1 call whose kernel's bounded wait ran out (synchronises each call).");
    m.def(
        "check_waits", []() { return check_waits_flag().load(); },
        "Whether K1 calls check the kernels' bounded waits (K1_CHECK_WAITS / set_check_waits).");
}
