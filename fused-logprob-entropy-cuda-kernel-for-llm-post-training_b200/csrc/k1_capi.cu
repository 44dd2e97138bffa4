// k1_capi.cu -- extern "C" entry points of libk1_b200.so (declared in
// include/k1_logprob.h): argument validation, launch configuration, error reporting.
//
// The reference's host dispatch (csrc/fused_logprob.cu:284-458) validates torch
// tensors with TORCH_CHECK and launches one 256-thread block per row.  Here the
// validation is on raw pointers / sizes (the torch-facing checks live in the binding
// layer, k1_torch_binding.cpp), and every kernel gets a grid of
// (SM count) x (resident blocks per SM) blocks that split the flattened work evenly.
#include <algorithm>
#include <vector>
#include <tuple>
#include <cmath>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <type_traits>
#include <utility>

#include "k1_fwd_sm.cuh"
#include "k1_lmhead.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#ifndef K1_PDL
#define K1_PDL 1
#endif

// Launch with programmatic stream serialization (see pdl_wait / pdl_trigger): the grid
// may be scheduled while the previous kernel of the stream drains; it waits for that
// kernel's completion on the device before touching memory.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), int64_t grid, int block, size_t smem,
                   cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = K1_PDL ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(K1_ERR_CUDA, "%s: kernel launch failed: %s", what, cudaGetErrorString(e));
    return K1_OK;
}

#ifndef K1_FWD_THREADS
#define K1_FWD_THREADS 256
#endif
constexpr int kThreads = 256;                  // backward (register path), naive helpers
constexpr int kFwdThreads = K1_FWD_THREADS;    // forward block size
constexpr int kUnroll = K1_FWD_UNROLL;      // 16-byte vectors per thread and chunk (forward)
constexpr int kUnrollBwd = K1_BWD_UNROLL;   // 16-byte vectors per thread and chunk (backward)
#ifndef K1_RING
#define K1_RING 1
#endif
#ifndef K1_RING_FWD
#define K1_RING_FWD 0
#endif
#ifndef K1_RING_WARPS
#define K1_RING_WARPS 16
#endif
#ifndef K1_RING_STAGES
#define K1_RING_STAGES 4
#endif
#ifndef K1_RING_BYTES
#define K1_RING_BYTES 16384
#endif
constexpr bool kRing = K1_RING != 0;        // bulk-copy ring backward on the vector path
constexpr bool kRingFwd = K1_RING_FWD != 0; // bulk-copy ring forward on the vector path
constexpr int kRingWarps = K1_RING_WARPS;   // consumer warps per block (+1 producer warp)
constexpr int kRingStages = K1_RING_STAGES;
constexpr int kRingBytes = K1_RING_BYTES;   // bytes per ring stage
constexpr int kMaxDevices = 64;
constexpr int kMaxBlocksPerSm = 8;   // grid cap
// Forward dynamic tail: the last (1 - K1_FWD_STATIC_NUM / K1_FWD_STATIC_DEN) of the units
// are cut into chunks that blocks take once their static piece is done -- whole rows,
// at least K1_FWD_TAIL_ROWS per chunk (more when the owners would not fit the workspace),
// when that is > 0, else K1_FWD_DYN_CHUNKS equal chunks per block.  Only when the launch
// has at least K1_FWD_TAIL_MIN_ROWS rows per block: with fewer, the tail's extra segments
// cost more than the balance gains.  Measured on B200 (bf16, V = 152064): 1024 and 2048
// rows unchanged (no tail), 4096 rows -3.6 %, 8192 rows -5.8 %, 16384 rows -5.6 %.
#ifndef K1_FWD_STATIC_NUM
#define K1_FWD_STATIC_NUM 3
#endif
#ifndef K1_FWD_STATIC_DEN
#define K1_FWD_STATIC_DEN 4
#endif
#ifndef K1_FWD_DYN_CHUNKS
#define K1_FWD_DYN_CHUNKS 2
#endif
#ifndef K1_FWD_TAIL_ROWS
#define K1_FWD_TAIL_ROWS 1
#endif
#ifndef K1_FWD_TAIL_MIN_ROWS
#define K1_FWD_TAIL_MIN_ROWS 4
#endif
constexpr int kMaxOwnersPerSm = 32;  // static pieces + dynamic chunks; sizes the workspace
// Forward row groups (k1_fwd_rows_kernel): the smallest group of 1, 2 or 4 warps that gets
// at least K1_FWD_ROWS_MIN whole rows from the queue; else whole-block groups when each
// block gets at least K1_FWD_ROWS_BLOCK_MIN rows; else the block kernel, which splits rows
// between blocks (and takes the scalar path).  Measured on B200 (forward, bf16, us, block
// kernel -> row groups): 1024 x 152064 71.8 -> 67.9, 2048 x 152064 124.9 -> 110.9,
// 16384 x 151936 809 -> 766, 32768 x 32000 446 -> 354, 65536 x 4096 362 -> 111.
// 0 disables.
#ifndef K1_FWD_ROWS
#define K1_FWD_ROWS 1
#endif
#ifndef K1_FWD_ROWS_MIN
#define K1_FWD_ROWS_MIN 3
#endif
#ifndef K1_FWD_ROWS_BLOCK_MIN
#define K1_FWD_ROWS_BLOCK_MIN 2
#endif
#ifndef K1_FWD_ROWS_FORCE_GT
#define K1_FWD_ROWS_FORCE_GT 0  // measurement builds only: always use this group size
#endif
// Forward, one block per SM (k1_fwd_sm_kernel, vector path): at least one row per SM,
// rows of at least K1_FWD_SM_MIN_CHUNKS chunks (32 x 8 vectors), at most
// K1_FWD_SM_MAX_CHUNKS_PER_SM chunks per SM in all.  Beyond that the row groups' whole
// rows cost less than the grabs' merges.  Measured on B200 (forward, bf16, us, row groups
// or split rows -> one block per SM): 148 x 152064 23.6 -> 19.5, 1024 x 152064 68.6 ->
// 62.5, 512 x 65536 29.7 -> 21.5, 4096 x 131072 179.2 -> 173.1, 16384 x 65536 353 -> 327;
// 16384 x 256000 1256 -> 1320 and 8192 x 32000 105.5 -> 107.5 stay on row groups.
// 0 disables.
#ifndef K1_FWD_SM
#define K1_FWD_SM 1
#endif
#ifndef K1_FWD_SM_WARPS
#define K1_FWD_SM_WARPS 16
#endif
#ifndef K1_FWD_SM_MIN_CHUNKS
#define K1_FWD_SM_MIN_CHUNKS 24
#endif
#ifndef K1_FWD_SM_MAX_CHUNKS_PER_SM
#define K1_FWD_SM_MAX_CHUNKS_PER_SM 8192
#endif
// The scaled forward (temperature folded in) does more arithmetic per logit: 24 warps
// without the prefetch buffer beat 16 with it (config 2 scaled 73.7 -> 69.7 us).  Warp
// count and prefetch do not change a grab's arithmetic, so the scaled forward keeps the
// same bits as the unscaled one on logits divided beforehand; for that, both select the
// kernel by the same rule.
#ifndef K1_FWD_SM_WARPS_SCALED
#define K1_FWD_SM_WARPS_SCALED 24
#endif
#ifndef K1_SM_PREFETCH_SCALED
#define K1_SM_PREFETCH_SCALED 0
#endif
template <bool SCALED>
constexpr int kSmWarps = SCALED ? K1_FWD_SM_WARPS_SCALED : K1_FWD_SM_WARPS;
template <bool SCALED>
constexpr bool kSmPrefetch = SCALED ? (K1_SM_PREFETCH_SCALED != 0) : (K1_SM_PREFETCH != 0);
constexpr int64_t kMinUnitsPerBlockVec = (int64_t)kThreads * kUnroll;
constexpr int64_t kMinUnitsPerBlockScalar = (int64_t)kThreads * 64;

int elem_size(int dtype) { return dtype == K1_DTYPE_F32 ? 4 : 2; }

int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return fail(K1_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (*dev < 0 || *dev >= kMaxDevices) return fail(K1_ERR_CUDA, "device ordinal %d out of range", *dev);
    return K1_OK;
}

int sm_count(int dev, int* out) {
    static std::atomic<int> cache[kMaxDevices];
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return fail(K1_ERR_CUDA, "cudaDeviceGetAttribute(SM count): %s", cudaGetErrorString(e));
        cache[dev].store(v, std::memory_order_relaxed);
    }
    *out = v;
    return K1_OK;
}

// Resident blocks per SM of one kernel instance, cached per (device, kernel).  Kernels
// with more than 48 KB of dynamic shared memory get the opt-in attribute set here, once
// per device.
template <typename Kernel>
int blocks_per_sm(Kernel kernel, int dev, int threads, size_t smem, int* out) {
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, int> cache;
    const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return K1_OK;
        }
    }
    cudaError_t e = cudaSuccess;
    if (smem > 0) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess)
            return fail(K1_ERR_CUDA, "cudaFuncSetAttribute(smem): %s", cudaGetErrorString(e));
    }
    int v = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, threads, smem);
    if (e != cudaSuccess) return fail(K1_ERR_CUDA, "occupancy query: %s", cudaGetErrorString(e));
    if (v < 1) v = 1;
    if (v > kMaxBlocksPerSm) v = kMaxBlocksPerSm;
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = v;
    *out = v;
    return K1_OK;
}

struct Rows {
    int64_t n_rows, vocab, inner_rows, inner_stride, outer_stride;
};

int check_rows(const char* fn, const Rows& L) {
    if (L.n_rows < 0) return fail(K1_ERR_INVALID_ARGUMENT, "%s: n_rows must be >= 0", fn);
    if (L.vocab < 1) return fail(K1_ERR_INVALID_ARGUMENT, "%s: vocab must be >= 1", fn);
    if (L.inner_rows < 1 || L.n_rows % L.inner_rows != 0)
        return fail(K1_ERR_INVALID_ARGUMENT,
                    "%s: inner_rows (%lld) must be >= 1 and divide n_rows (%lld)", fn,
                    (long long)L.inner_rows, (long long)L.n_rows);
    if (L.inner_stride < 0 || L.outer_stride < 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: strides must be >= 0", fn);
    return K1_OK;
}

// Whether every row starts on a 16-byte boundary and holds whole 16-byte vectors.
bool vector_ok(const void* base, int es, const Rows& L) {
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
    if ((L.vocab * es) % 16 != 0) return false;
    if (L.inner_rows > 1 && (L.inner_stride * es) % 16 != 0) return false;
    if (L.n_rows > L.inner_rows && (L.outer_stride * es) % 16 != 0) return false;
    return true;
}

// Whether every logits row and its gradient row have the same address modulo 16 bytes
// (then both can be peeled at the same element: see peel in k1_kernels.cuh).
bool peel_congruent(const void* x, const void* d, int es, const Rows& L, const Rows& D) {
    const int64_t base = (int64_t)(reinterpret_cast<uintptr_t>(x) % 16) -
                         (int64_t)(reinterpret_cast<uintptr_t>(d) % 16);
    if (base != 0) return false;
    if (L.inner_rows > 1 && ((L.inner_stride - D.inner_stride) * es) % 16 != 0) return false;
    if (L.n_rows > L.inner_rows && ((L.outer_stride - D.outer_stride) * es) % 16 != 0)
        return false;
    return true;
}

k1::RowLayout layout_of(const Rows& L) {
    k1::RowLayout r;
    r.inner_rows = L.inner_rows;
    r.inner_stride = L.inner_stride;
    r.outer_stride = L.outer_stride;
    return r;
}

// Workspace layout: 2 row partials per owner, one ticket per owner, 2 dynamic-tail
// counters (next chunk, blocks done), padding.
size_t max_owners(int sms) { return (size_t)sms * kMaxOwnersPerSm; }
size_t workspace_bytes_for(int sms) {
    const size_t o = max_owners(sms);
    return 2 * o * sizeof(k1::RowPartial) + o * sizeof(unsigned) + 2 * sizeof(unsigned) + 64;
}
// Bytes at the end of the workspace that must be zero before a call (tickets, counters).
size_t workspace_zero_offset(int sms) { return 2 * max_owners(sms) * sizeof(k1::RowPartial); }
size_t workspace_zero_bytes(int sms) { return max_owners(sms) * sizeof(unsigned) + 2 * sizeof(unsigned); }

template <typename Kernel>
int grid_for(Kernel kernel, int dev, int64_t total, int64_t min_units, int64_t* grid,
             int threads = kThreads, size_t smem = 0) {
    int sms = 0, occ = 0;
    int rc = sm_count(dev, &sms);
    if (rc) return rc;
    rc = blocks_per_sm(kernel, dev, threads, smem, &occ);
    if (rc) return rc;
    int64_t g = (int64_t)sms * occ;
    int64_t need = (total + min_units - 1) / min_units;
    if (need < 1) need = 1;
    if (g > need) g = need;
    if (g > total) g = total;
    if (g < 1) g = 1;
    *grid = g;
    return K1_OK;
}

template <typename T, bool SHARD, bool SCALED = false>
int launch_forward(const char* fn, const void* logits, const Rows& L, int64_t col_offset,
                   const int64_t* targets, float* logprob, float* entropy, float* lse,
                   k1_partial* partials, void* workspace, size_t workspace_bytes,
                   cudaStream_t stream, float scale = 1.f) {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    int sms = 0;
    rc = sm_count(dev, &sms);
    if (rc) return rc;
    if (workspace == nullptr || workspace_bytes < workspace_bytes_for(sms))
        return fail(K1_ERR_WORKSPACE, "%s: workspace of %zu bytes required (got %zu)", fn,
                    workspace_bytes_for(sms), workspace == nullptr ? (size_t)0 : workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: workspace must be 16-byte aligned", fn);

    const int es = (int)sizeof(T);
    const bool vec = vector_ok(logits, es, L);
    k1::FwdParams p;
    p.logits = logits;
    p.n_rows = L.n_rows;
    p.vocab = L.vocab;
    p.lay = layout_of(L);
    p.vpr = vec ? L.vocab / k1::DT<T>::kEPV : L.vocab;
    p.total = L.n_rows * p.vpr;
    p.col_offset = col_offset;
    p.targets = targets;
    p.logprob = logprob;
    p.entropy = entropy;
    p.lse = lse;
    p.partials = partials;
    p.scale = SCALED ? scale : 1.f;
    const size_t omax = max_owners(sms);
    p.ws_part = reinterpret_cast<k1::RowPartial*>(workspace);
    p.ws_ticket = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(workspace) +
                                              2 * omax * sizeof(k1::RowPartial));
    p.ws_dyn = p.ws_ticket + omax;
    p.split = p.total;
    p.n_dyn = 0;
    p.dyn_units = 1;
    // dynamic tail for the register-path kernel (see K1_FWD_TAIL_*); every owner non-empty
    auto plan_tail = [&](int64_t grid) {
        if (L.n_rows < (int64_t)K1_FWD_TAIL_MIN_ROWS * grid) return;
        int64_t split = p.total / K1_FWD_STATIC_DEN * K1_FWD_STATIC_NUM +
                        p.total % K1_FWD_STATIC_DEN * K1_FWD_STATIC_NUM / K1_FWD_STATIC_DEN;
        int64_t csize;
        if (K1_FWD_TAIL_ROWS > 0) {
            split = split / p.vpr * p.vpr;  // the tail starts on a row
            const int64_t tail_rows = (p.total - split) / p.vpr;
            const int64_t room = (int64_t)omax - grid;  // owners the workspace still holds
            if (room < 1) return;
            int64_t rows = K1_FWD_TAIL_ROWS;
            if (tail_rows > rows * room) rows = (tail_rows + room - 1) / room;
            csize = rows * p.vpr;
        } else {
            if (K1_FWD_DYN_CHUNKS <= 0) return;
            const int64_t want = grid * K1_FWD_DYN_CHUNKS;
            csize = (p.total - split + want - 1) / want;
        }
        if (split < grid || split >= p.total || csize < 1) return;
        const int64_t D = (p.total - split + csize - 1) / csize;
        if ((size_t)(grid + D) > omax) return;
        p.split = split;
        p.n_dyn = D;
        p.dyn_units = csize;
    };
    int64_t grid = 1;
    // (build-time alternatives are only instantiated when selected)
    if constexpr (kRingFwd && !SCALED) {
        if (vec) {
            auto kern = k1::k1_fwd_ring_kernel<T, kRingWarps, kRingStages, kRingBytes, SHARD>;
            const int threads = (kRingWarps + 1) * 32;
            const size_t smem = (size_t)kRingStages * kRingBytes;
            rc = grid_for(kern, dev, p.total, kMinUnitsPerBlockVec, &grid, threads, smem);
            if (rc) return rc;
            launch(kern, grid, threads, smem, stream, p);
            return check_launch(fn);
        }
    }
    if (K1_FWD_SM && vec) {
        const int64_t cpr = (p.vpr + 32 * kUnroll - 1) / (32 * kUnroll);
        if (cpr >= K1_FWD_SM_MIN_CHUNKS && L.n_rows >= sms && p.vpr < (int64_t)1 << 30 &&
            L.n_rows * cpr <= (int64_t)K1_FWD_SM_MAX_CHUNKS_PER_SM * sms &&
            L.n_rows <= (int64_t)sms << 20) {
            constexpr int nw = kSmWarps<SCALED>;
            auto kern = k1::k1_fwd_sm_kernel<T, nw, kUnroll, SHARD, SCALED, kSmPrefetch<SCALED>>;
            const size_t smem = sizeof(k1::SmFwdSmem);
            int occ = 0;
            rc = blocks_per_sm(kern, dev, nw * 32, smem, &occ);
            if (rc) return rc;
            launch(kern, std::min<int64_t>(sms, L.n_rows), nw * 32, smem, stream, p);
            return check_launch(fn);
        }
    }
    if (K1_FWD_ROWS) {
        // row groups: the smallest group that still gets K1_FWD_ROWS_MIN rows (any
        // alignment: rows that are not whole vectors are peeled, see fwd_stream_peeled)
        auto rows_launch = [&](auto kern, int gt, int min_rows) -> int {
            int64_t g = 1;
            int r = grid_for(kern, dev, p.total, 1, &g, 256);
            if (r) return r;
            const int64_t groups = g * (256 / gt);
            if (K1_FWD_ROWS_FORCE_GT != 0) {
                if (gt != K1_FWD_ROWS_FORCE_GT) return -1;
            } else if (L.n_rows < (int64_t)min_rows * groups) {
                return -1;
            }
            launch(kern, g, 256, 0, stream, p);
            return check_launch(fn);
        };
        auto try_all = [&](auto vec_tag) -> int {
            constexpr bool V = decltype(vec_tag)::value;
            constexpr int kMin = K1_FWD_ROWS_MIN;
            int r = rows_launch(k1::k1_fwd_rows_kernel<T, 32, kUnroll, V, SHARD, SCALED>, 32, kMin);
            if (r < 0)
                r = rows_launch(k1::k1_fwd_rows_kernel<T, 64, kUnroll, V, SHARD, SCALED>, 64, kMin);
            if (r < 0)
                r = rows_launch(k1::k1_fwd_rows_kernel<T, 128, kUnroll, V, SHARD, SCALED>, 128, kMin);
            if (r < 0)
                r = rows_launch(k1::k1_fwd_rows_kernel<T, 256, kUnroll, V, SHARD, SCALED>, 256,
                                K1_FWD_ROWS_BLOCK_MIN);
            return r;
        };
        rc = vec ? try_all(std::true_type{}) : try_all(std::false_type{});
        if (rc >= 0) return rc;
    }
    if (vec) {
        auto kern = k1::k1_fwd_kernel<T, kFwdThreads, kUnroll, true, SHARD, SCALED>;
        rc = grid_for(kern, dev, p.total, kMinUnitsPerBlockVec, &grid, kFwdThreads);
        if (rc) return rc;
        plan_tail(grid);
        launch(kern, grid, kFwdThreads, 0, stream, p);
    } else {
        auto kern = k1::k1_fwd_kernel<T, kFwdThreads, kUnroll, false, SHARD, SCALED>;
        rc = grid_for(kern, dev, p.total, kMinUnitsPerBlockScalar, &grid, kFwdThreads);
        if (rc) return rc;
        plan_tail(grid);
        launch(kern, grid, kFwdThreads, 0, stream, p);
    }
    return check_launch(fn);
}

template <typename T, bool SCALED = false>
int launch_backward(const char* fn, const void* logits, const Rows& L, const Rows& D,
                    int64_t col_offset, const int64_t* targets, const float* lse,
                    const float* entropy, const float* g_logp, const float* g_ent,
                    const float* g_lse, void* d_logits, cudaStream_t stream, float scale = 1.f) {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    const int es = (int)sizeof(T);
    const bool vec = vector_ok(logits, es, L) && vector_ok(d_logits, es, D);
    k1::BwdParams p;
    p.logits = logits;
    p.dlogits = d_logits;
    p.n_rows = L.n_rows;
    p.vocab = L.vocab;
    p.lay = layout_of(L);
    p.dlay = layout_of(D);
    p.vpr = vec ? L.vocab / k1::DT<T>::kEPV : L.vocab;
    p.total = L.n_rows * p.vpr;
    p.col_offset = col_offset;
    p.targets = targets;
    p.lse = lse;
    p.entropy = entropy;
    p.g_logp = g_logp;
    p.g_ent = g_ent;
    p.g_lse = g_lse;
    p.scale = SCALED ? scale : 1.f;
    int64_t grid = 1;
    // (build-time alternatives are only instantiated when selected)
    if constexpr (kRing) {
        if (vec) {
            auto kern = k1::k1_bwd_ring_kernel<T, kRingWarps, kRingStages, kRingBytes, SCALED>;
            const int threads = (kRingWarps + 1) * 32;
            const size_t smem = (size_t)kRingStages * kRingBytes;
            rc = grid_for(kern, dev, p.total, kMinUnitsPerBlockVec, &grid, threads, smem);
            if (rc) return rc;
            launch(kern, grid, threads, smem, stream, p);
            return check_launch(fn);
        }
        if (peel_congruent(logits, d_logits, es, L, D)) {
            // rows that are not whole vectors: the ring over each segment's aligned interior
            auto kern = k1::k1_bwd_ring_kernel<T, kRingWarps, kRingStages, kRingBytes, SCALED, true>;
            const int threads = (kRingWarps + 1) * 32;
            const size_t smem = (size_t)kRingStages * kRingBytes;
            rc = grid_for(kern, dev, p.total, kMinUnitsPerBlockVec * k1::DT<T>::kEPV, &grid,
                          threads, smem);
            if (rc) return rc;
            launch(kern, grid, threads, smem, stream, p);
            return check_launch(fn);
        }
    } else {
        if (vec) {
            auto kern = k1::k1_bwd_kernel<T, kThreads, kUnrollBwd, true, SCALED>;
            rc = grid_for(kern, dev, p.total, kMinUnitsPerBlockVec, &grid);
            if (rc) return rc;
            launch(kern, grid, kThreads, 0, stream, p);
            return check_launch(fn);
        }
    }
    {
        auto kern = k1::k1_bwd_kernel<T, kThreads, kUnrollBwd, false, SCALED>;
        rc = grid_for(kern, dev, p.total, kMinUnitsPerBlockScalar, &grid);
        if (rc) return rc;
        launch(kern, grid, kThreads, 0, stream, p);
    }
    return check_launch(fn);
}

// ---------------------------------------------------------------------------------
// Allocation-free forward: its split-row scratch is this file-scope device array, so the
// entry point needs no workspace from the caller.  Every GPU that loads the library
// holds the array until the process exits.  Every call on a device shares it.
// ---------------------------------------------------------------------------------
constexpr size_t kStaticScratchBytes = 512 * 1024;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on device `dev`, looked up once per device with
// that device current (the symbol's name is only a host-side handle, not an address).
int static_scratch_ptr(int dev, void** out) {
    static std::mutex mu;
    static void* ptrs[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (ptrs[dev] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(K1_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s",
                        cudaGetErrorString(e));
        ptrs[dev] = p;
    }
    *out = ptrs[dev];
    return K1_OK;
}

// A logit scale (reciprocal sampling temperature) must be a positive finite number.
int check_scale(const char* fn, float scale) {
    if (!(scale > 0.f) || !(scale <= 3.402823466e38f))
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: scale must be positive and finite (got %g)", fn,
                    (double)scale);
    return K1_OK;
}

int check_common(const char* fn, const void* logits, int dtype, const Rows& L) {
    if (dtype != K1_DTYPE_F32 && dtype != K1_DTYPE_F16 && dtype != K1_DTYPE_BF16)
        return fail(K1_ERR_UNSUPPORTED_DTYPE, "%s: logits dtype must be bf16, fp16, or fp32", fn);
    int rc = check_rows(fn, L);
    if (rc) return rc;
    if (L.n_rows > 0 && logits == nullptr)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: logits is NULL", fn);
    if (reinterpret_cast<uintptr_t>(logits) % elem_size(dtype) != 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: logits not aligned to its element size", fn);
    return K1_OK;
}


// ---------------------------------------------------------------------------------------
// LM head fused with K1 (k1_lmhead.cuh): tensor maps, work split, launches
// ---------------------------------------------------------------------------------------
using TmapEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver, looked up through the runtime (no link-time
// dependency on libcuda).
int tmap_encoder(TmapEncodeFn* out) {
    static std::once_flag once;
    static TmapEncodeFn fn = nullptr;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<TmapEncodeFn>(f);
    });
    if (!fn) return fail(K1_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    *out = fn;
    return K1_OK;
}

// Row-major bf16 [rows, cols] matrix read in boxes of box_rows x 64 with 128-byte swizzle.
int make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows,
              const char* what) {
    TmapEncodeFn enc = nullptr;
    int rc = tmap_encoder(&enc);
    if (rc) return rc;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)k1::lmh::BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                     box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(K1_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed: %d", what, (int)r);
    return K1_OK;
}

// Units per row block: the number of runs the vocabulary tiles are cut into.  Chosen among
// runs of 1 to 32 tiles (the per-row partials kept within 64 MiB) so that the CTA with the
// most tiles (units are dealt round robin, in the kernel's unit order) has as few as
// possible, the fewest parts among equals; cached per shape.
int lmh_parts(int m_blocks, int tile_m, int n_tiles, int grid) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int>, int> cache;
    const auto key = std::make_tuple(m_blocks, tile_m, n_tiles, grid);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    int best = 1;
    int64_t best_max = INT64_MAX;
    const int64_t rows = (int64_t)m_blocks * tile_m;
    const int64_t cap = ((int64_t)64 << 20) / (rows * (int64_t)sizeof(k1::RowPartial));
    const int lo = std::max(1, (n_tiles + 31) / 32);
    const int hi = (int)std::max<int64_t>(lo, std::min<int64_t>(std::min(n_tiles, 2048), cap));
    std::vector<int64_t> load(grid);
    for (int np = lo; np <= hi; ++np) {
        std::fill(load.begin(), load.end(), 0);
        const int64_t units = (int64_t)m_blocks * np;
        // unit u -> part: the kernel's order (groups of GROUP_M row blocks, row block fastest)
        for (int64_t u = 0; u < units; ++u) {
            const int64_t per_group = (int64_t)k1::lmh::GROUP_M * np;
            const int64_t g = u / per_group, r = u - g * per_group;
            const int64_t rows_in_group = std::min<int64_t>(k1::lmh::GROUP_M, m_blocks - g * k1::lmh::GROUP_M);
            const int64_t part = r / rows_in_group;
            const int64_t tiles = (part + 1) * n_tiles / np - part * n_tiles / np;
            load[u % grid] += tiles;
        }
        const int64_t mx = *std::max_element(load.begin(), load.end());
        if (mx < best_max) {
            best_max = mx;
            best = np;
        }
    }
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = best;
    return best;
}

// CTA pairs (tcgen05.mma.cta_group::2, 256 x 256 tiles) or single CTAs (128 x 256).
#ifndef K1_LMH_PAIR
#define K1_LMH_PAIR 1
#endif

// Pairs that can be resident at once (a cluster of 2 CTAs of ~200 KB shared memory must
// fit on two SMs of one GPC): the persistent grid must not exceed it, or part of it would
// run only after the rest has finished.  Cached per device.
int lmh_pair_clusters(int dev, int* out) {
    static std::atomic<int> cache[kMaxDevices];
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        auto kern = k1::lmh::k1_lmhead_kernel<k1::lmh::STATS, false, true>;
        const int smem = k1::lmh::Geo<true>::SMEM;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return fail(K1_ERR_CUDA, "cudaFuncSetAttribute(smem): %s", cudaGetErrorString(e));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(k1::lmh::THREADS);
        cfg.dynamicSmemBytes = (size_t)smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
        if (e != cudaSuccess || n < 1)
            return fail(K1_ERR_CUDA, "cudaOccupancyMaxActiveClusters: %s (%d)", cudaGetErrorString(e), n);
        v = n;
        cache[dev].store(v, std::memory_order_relaxed);
    }
    *out = v;
    return K1_OK;
}

struct LmhShape {
    int m_blocks, n_tiles, k_blocks, grid, n_parts;  // grid: CTAs, or pairs with PAIR
    bool pair;
};

int lmh_shape(int64_t n_rows, int64_t hidden, int64_t vocab, int dev, LmhShape* sh) {
    int sms = 0;
    int rc = sm_count(dev, &sms);
    if (rc) return rc;
    sh->pair = K1_LMH_PAIR != 0 && sms >= 2;
    const int tile_m = k1::lmh::BM * (sh->pair ? 2 : 1);
    sh->m_blocks = (int)((n_rows + tile_m - 1) / tile_m);
    sh->n_tiles = (int)((vocab + k1::lmh::BN - 1) / k1::lmh::BN);
    const int kb = sh->pair ? k1::lmh::Geo<true>::KB : k1::lmh::Geo<false>::KB;  // K per stage
    sh->k_blocks = (int)((hidden + kb - 1) / kb);
    const int64_t max_units = (int64_t)sh->m_blocks * sh->n_tiles;
    int slots = sms;
    if (sh->pair) {
        rc = lmh_pair_clusters(dev, &slots);
        if (rc) return rc;
    }
    sh->grid = (int)std::min<int64_t>(slots, max_units);
    sh->n_parts = lmh_parts(sh->m_blocks, tile_m, sh->n_tiles, sh->grid);
    return K1_OK;
}

// Partials [n_parts][n_rows], target logits [n_rows], the finished-unit counter.
size_t lmh_workspace_bytes(int64_t n_rows, const LmhShape& sh) {
    return (size_t)sh.n_parts * (size_t)n_rows * sizeof(k1::RowPartial) + (size_t)n_rows * sizeof(float) + 256;
}

int lmh_check(const char* fn, const void* hidden, const void* weight, int64_t n_rows,
              int64_t hidden_dim, int64_t vocab) {
    if (!hidden || !weight) return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL hidden or weight", fn);
    if (n_rows < 0 || vocab < 1 || hidden_dim < 1)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: bad sizes (n_rows %lld, hidden %lld, vocab %lld)", fn,
                    (long long)n_rows, (long long)hidden_dim, (long long)vocab);
    if (hidden_dim % 8 != 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: hidden size must be a multiple of 8 (got %lld)",
                    fn, (long long)hidden_dim);
    if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(weight)) % 16 != 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: hidden and weight must be 16-byte aligned", fn);
    if (n_rows > ((int64_t)1 << 31) - k1::lmh::BM || vocab > ((int64_t)1 << 31) - k1::lmh::BN)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: n_rows and vocab must stay below 2^31", fn);
    return K1_OK;
}

template <int MODE>
int lmh_launch(const char* fn, const void* hidden, const void* weight, int64_t n_rows,
               int64_t hidden_dim, int64_t vocab, float scale, k1::lmh::Params p,
               const LmhShape& sh, cudaStream_t s) {
    CUtensorMap th, tw;
    int rc = make_tmap(&th, hidden, n_rows, hidden_dim, k1::lmh::BM, "hidden");
    if (rc) return rc;
    rc = make_tmap(&tw, weight, vocab, hidden_dim, sh.pair ? k1::lmh::BN / 2 : k1::lmh::BN, "weight");
    if (rc) return rc;
    p.n_rows = n_rows;
    p.vocab = vocab;
    p.k_blocks = sh.k_blocks;
    p.m_blocks = sh.m_blocks;
    p.n_tiles = sh.n_tiles;
    p.n_parts = sh.n_parts;
    p.units = sh.m_blocks * sh.n_parts;
    p.scale = scale;
    const bool scaled = scale != 1.f;
    int dev = 0;
    rc = current_device(&dev);
    if (rc) return rc;
    // Launched without programmatic dependence, so it never shares an SM with the previous
    // kernel's blocks: the kernel allocates all of an SM's tensor memory.
    auto go = [&](auto kern, bool pair) -> int {
        const int smem = pair ? k1::lmh::Geo<true>::SMEM : k1::lmh::Geo<false>::SMEM;
        int occ = 0;
        int r = blocks_per_sm(kern, dev, k1::lmh::THREADS, (size_t)smem, &occ);
        if (r) return r;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(sh.grid * (pair ? 2 : 1)));
        cfg.blockDim = dim3(k1::lmh::THREADS);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = pair ? 2 : 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pair ? 1 : 0;
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, th, tw, p);
        if (e != cudaSuccess) return fail(K1_ERR_CUDA, "%s: launch failed: %s", fn, cudaGetErrorString(e));
        return K1_OK;
    };
    if (sh.pair)
        rc = scaled ? go(k1::lmh::k1_lmhead_kernel<MODE, true, true>, true)
                    : go(k1::lmh::k1_lmhead_kernel<MODE, false, true>, true);
    else
        rc = scaled ? go(k1::lmh::k1_lmhead_kernel<MODE, true, false>, false)
                    : go(k1::lmh::k1_lmhead_kernel<MODE, false, false>, false);
    if (rc) return rc;
    return check_launch(fn);
}
// The LM head's forward: the tensor-core kernel (statistics, or statistics + z), then the
// merge of the per-unit partials into either the finished rows (logprob, entropy, lse) or,
// for a vocabulary shard, each row's k1_partial.  col_offset: the global id of the weight's
// first row (0 for a whole vocabulary).
int lmh_forward(const char* fn, const void* hidden, const void* weight, int64_t n_rows,
                int64_t hidden_dim, int64_t vocab, int64_t col_offset, float scale,
                const int64_t* targets, float* logprob, float* entropy, float* lse,
                k1_partial* partials, void* logits_out, int64_t logits_stride, void* workspace,
                size_t workspace_bytes, void* stream) {
    int rc = lmh_check(fn, hidden, weight, n_rows, hidden_dim, vocab);
    if (rc) return rc;
    if (n_rows == 0) return K1_OK;
    if (!targets) return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets or output pointer", fn);
    if (!(scale > 0.f) || !std::isfinite(scale))
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: scale must be positive and finite", fn);
    if (logits_out && logits_stride < vocab)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: logits_stride must be >= vocab", fn);
    int dev = 0;
    rc = current_device(&dev);
    if (rc) return rc;
    LmhShape sh;
    rc = lmh_shape(n_rows, hidden_dim, vocab, dev, &sh);
    if (rc) return rc;
    const size_t need = lmh_workspace_bytes(n_rows, sh);
    if (!workspace || workspace_bytes < need)
        return fail(K1_ERR_WORKSPACE, "%s: workspace of %zu bytes required (got %zu)", fn, need,
                    workspace ? workspace_bytes : (size_t)0);
    if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: workspace must be 16-byte aligned", fn);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    k1::lmh::Params p = {};
    p.col_offset = col_offset;
    p.targets = targets;
    p.part = reinterpret_cast<k1::RowPartial*>(workspace);
    p.xt = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                    (size_t)sh.n_parts * n_rows * sizeof(k1::RowPartial));
    p.out = reinterpret_cast<__nv_bfloat16*>(logits_out);
    p.out_stride = logits_stride;
    {
        // the unit counter after the partials and target logits (16-byte aligned)
        const size_t off = ((size_t)sh.n_parts * n_rows * sizeof(k1::RowPartial) +
                            (size_t)n_rows * sizeof(float) + 15) & ~(size_t)15;
        p.done = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(workspace) + off);
        cudaError_t e = cudaMemsetAsync(p.done, 0, sizeof(unsigned), s);
        if (e != cudaSuccess) return fail(K1_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
    }
    rc = logits_out ? lmh_launch<k1::lmh::STORE>(fn, hidden, weight, n_rows, hidden_dim, vocab,
                                                 scale, p, sh, s)
                    : lmh_launch<k1::lmh::STATS>(fn, hidden, weight, n_rows, hidden_dim, vocab,
                                                 scale, p, sh, s);
    if (rc) return rc;
    const int threads = 256;
    const unsigned blocks = (unsigned)((n_rows + threads - 1) / threads);
    const unsigned expected =
        (unsigned)(sh.m_blocks * sh.n_parts) * k1::lmh::EPI_WARPS * (sh.pair ? 2u : 1u);
    if (partials)
        k1::lmh::k1_lmhead_shard_merge_kernel<<<blocks, threads, 0, s>>>(
            p.part, p.xt, targets, n_rows, vocab, col_offset, sh.n_parts, p.done, expected, partials);
    else
        k1::lmh::k1_lmhead_merge_kernel<<<blocks, threads, 0, s>>>(
            p.part, p.xt, targets, n_rows, vocab, sh.n_parts, p.done, expected, logprob, entropy, lse);
    return check_launch(fn);
}

// The LM head's backward to the logits (GRAD mode), for a whole vocabulary or a shard.
int lmh_backward(const char* fn, const void* hidden, const void* weight, int64_t n_rows,
                 int64_t hidden_dim, int64_t vocab, int64_t col_offset, float scale,
                 const int64_t* targets, const float* lse, const float* entropy,
                 const float* g_logp, const float* g_ent, const float* g_lse, void* d_logits,
                 int64_t d_stride, void* stream) {
    int rc = lmh_check(fn, hidden, weight, n_rows, hidden_dim, vocab);
    if (rc) return rc;
    if (n_rows == 0) return K1_OK;
    if (!targets || !lse || !entropy || !d_logits)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets, lse, entropy or d_logits", fn);
    if (!(scale > 0.f) || !std::isfinite(scale))
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: scale must be positive and finite", fn);
    if (d_stride < vocab) return fail(K1_ERR_INVALID_ARGUMENT, "%s: d_stride must be >= vocab", fn);
    int dev = 0;
    rc = current_device(&dev);
    if (rc) return rc;
    LmhShape sh;
    rc = lmh_shape(n_rows, hidden_dim, vocab, dev, &sh);
    if (rc) return rc;
    k1::lmh::Params p = {};
    p.col_offset = col_offset;
    p.targets = targets;
    p.lse = lse;
    p.entropy = entropy;
    p.g_logp = g_logp;
    p.g_ent = g_ent;
    p.g_lse = g_lse;
    p.out = reinterpret_cast<__nv_bfloat16*>(d_logits);
    p.out_stride = d_stride;
    return lmh_launch<k1::lmh::GRAD>(fn, hidden, weight, n_rows, hidden_dim, vocab, scale, p, sh,
                                     reinterpret_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" {

const char* k1_last_error(void) { return g_last_error.c_str(); }

// Reads (and clears) the bulk-copy ring's timeout word on the current device; blocks
// until prior work on the device finished.  0 = no bounded wait ran out.
int k1_ring_status(unsigned* out) {
    unsigned v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, k1::k1_ring_error, sizeof v);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(k1::k1_ring_error, &zero, sizeof zero);
    if (e != cudaSuccess) return fail(K1_ERR_CUDA, "k1_ring_status: %s", cudaGetErrorString(e));
    if (out) *out = v;
    return K1_OK;
}

int k1_abi_version(void) { return K1_ABI_VERSION; }

size_t k1_forward_workspace_bytes(int64_t n_rows, int64_t vocab, int dtype, int device) {
    (void)n_rows;
    (void)vocab;
    (void)dtype;
    if (device < 0 || device >= kMaxDevices) return 0;
    int sms = 0;
    if (sm_count(device, &sms) != K1_OK) return 0;
    return workspace_bytes_for(sms);
}

int k1_fused_logprob_entropy_v1(const void* logits, int dtype, int64_t n_rows, int64_t vocab,
                                int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                                const int64_t* targets, float* logprob, float* entropy,
                                float* lse, void* workspace, size_t workspace_bytes,
                                void* stream) {
    static const char* fn = "k1_fused_logprob_entropy_v1";
    Rows L{n_rows, vocab, inner_rows, inner_stride, outer_stride};
    int rc = check_common(fn, logits, dtype, L);
    if (rc) return rc;
    if (n_rows == 0) return K1_OK;
    if (!targets || !logprob || !entropy || !lse)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets or output pointer", fn);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (dtype) {
        case K1_DTYPE_BF16:
            return launch_forward<__nv_bfloat16, false>(fn, logits, L, 0, targets, logprob, entropy,
                                                        lse, nullptr, workspace, workspace_bytes, s);
        case K1_DTYPE_F16:
            return launch_forward<__half, false>(fn, logits, L, 0, targets, logprob, entropy, lse,
                                                 nullptr, workspace, workspace_bytes, s);
        default:
            return launch_forward<float, false>(fn, logits, L, 0, targets, logprob, entropy, lse,
                                                nullptr, workspace, workspace_bytes, s);
    }
}

int k1_fused_logprob_entropy_v1_noalloc(const void* logits, int dtype, int64_t n_rows,
                                        int64_t vocab, int64_t inner_rows, int64_t inner_stride,
                                        int64_t outer_stride, const int64_t* targets,
                                        float* logprob, float* entropy, float* lse,
                                        void* stream) {
    static const char* fn = "k1_fused_logprob_entropy_v1_noalloc";
    Rows L{n_rows, vocab, inner_rows, inner_stride, outer_stride};
    int rc = check_common(fn, logits, dtype, L);
    if (rc) return rc;
    if (n_rows == 0) return K1_OK;
    if (!targets || !logprob || !entropy || !lse)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets or output pointer", fn);
    int dev = 0, sms = 0;
    rc = current_device(&dev);
    if (rc) return rc;
    rc = sm_count(dev, &sms);
    if (rc) return rc;
    // The scratch this device needs grows with its SM count, not with the problem size.
    const size_t need = workspace_bytes_for(sms);
    if (need > kStaticScratchBytes)
        return fail(K1_ERR_WORKSPACE,
                    "%s: this device (%d SMs) needs %zu bytes of scratch; the static scratch "
                    "holds at most %zu bytes",
                    fn, sms, need, kStaticScratchBytes);
    void* ws = nullptr;
    rc = static_scratch_ptr(dev, &ws);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // The tickets must start at zero; the previous call may not have left them so (it
    // may still be running on another stream, which is a documented race, or have been
    // interrupted).  Clearing is stream-ordered and allocates nothing.
    cudaError_t e = cudaMemsetAsync(reinterpret_cast<char*>(ws) + workspace_zero_offset(sms), 0,
                                    workspace_zero_bytes(sms), s);
    if (e != cudaSuccess)
        return fail(K1_ERR_CUDA, "%s: clearing the static scratch: %s", fn, cudaGetErrorString(e));
    switch (dtype) {
        case K1_DTYPE_BF16:
            return launch_forward<__nv_bfloat16, false>(fn, logits, L, 0, targets, logprob, entropy,
                                                        lse, nullptr, ws, kStaticScratchBytes, s);
        case K1_DTYPE_F16:
            return launch_forward<__half, false>(fn, logits, L, 0, targets, logprob, entropy, lse,
                                                 nullptr, ws, kStaticScratchBytes, s);
        default:
            return launch_forward<float, false>(fn, logits, L, 0, targets, logprob, entropy, lse,
                                                nullptr, ws, kStaticScratchBytes, s);
    }
}

int k1_fused_logprob_entropy_naive(const void* logits, int dtype, int64_t n_rows, int64_t vocab,
                                   int64_t inner_rows, int64_t inner_stride,
                                   int64_t outer_stride, const int64_t* targets,
                                   float* logprob, float* entropy, float* lse, void* stream) {
    static const char* fn = "k1_fused_logprob_entropy_naive";
    Rows L{n_rows, vocab, inner_rows, inner_stride, outer_stride};
    int rc = check_common(fn, logits, dtype, L);
    if (rc) return rc;
    if (n_rows == 0) return K1_OK;
    if (!targets || !logprob || !entropy || !lse)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets or output pointer", fn);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int threads = 128;
    const int64_t blocks = (n_rows + threads - 1) / threads;
    k1::RowLayout lay = layout_of(L);
    switch (dtype) {
        case K1_DTYPE_BF16:
            launch(k1::k1_naive_kernel<__nv_bfloat16>, blocks, threads, 0, s,
                   reinterpret_cast<const __nv_bfloat16*>(logits), n_rows, vocab, lay, targets,
                   logprob, entropy, lse);
            break;
        case K1_DTYPE_F16:
            launch(k1::k1_naive_kernel<__half>, blocks, threads, 0, s,
                   reinterpret_cast<const __half*>(logits), n_rows, vocab, lay, targets, logprob,
                   entropy, lse);
            break;
        default:
            launch(k1::k1_naive_kernel<float>, blocks, threads, 0, s,
                   reinterpret_cast<const float*>(logits), n_rows, vocab, lay, targets, logprob,
                   entropy, lse);
            break;
    }
    return check_launch(fn);
}

static int backward_impl(const char* fn, const void* logits, int dtype, int64_t n_rows,
                         int64_t vocab, int64_t inner_rows, int64_t inner_stride,
                         int64_t outer_stride, int64_t col_offset, const int64_t* targets,
                         const float* lse, const float* entropy, const float* g_logp,
                         const float* g_ent, const float* g_lse, void* d_logits,
                         int64_t d_inner_stride, int64_t d_outer_stride, void* stream,
                         float scale = 1.f) {
    Rows L{n_rows, vocab, inner_rows, inner_stride, outer_stride};
    Rows D{n_rows, vocab, inner_rows, d_inner_stride, d_outer_stride};
    int rc = check_common(fn, logits, dtype, L);
    if (rc) return rc;
    rc = check_rows(fn, D);
    if (rc) return rc;
    if (n_rows == 0) return K1_OK;
    if (!targets || !lse || !entropy || !d_logits)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets, lse, entropy or d_logits", fn);
    if (reinterpret_cast<uintptr_t>(d_logits) % elem_size(dtype) != 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: d_logits not aligned to its element size", fn);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (scale != 1.f) {
        switch (dtype) {
            case K1_DTYPE_BF16:
                return launch_backward<__nv_bfloat16, true>(fn, logits, L, D, col_offset, targets,
                                                            lse, entropy, g_logp, g_ent, g_lse,
                                                            d_logits, s, scale);
            case K1_DTYPE_F16:
                return launch_backward<__half, true>(fn, logits, L, D, col_offset, targets, lse,
                                                     entropy, g_logp, g_ent, g_lse, d_logits, s,
                                                     scale);
            default:
                return launch_backward<float, true>(fn, logits, L, D, col_offset, targets, lse,
                                                    entropy, g_logp, g_ent, g_lse, d_logits, s,
                                                    scale);
        }
    }
    switch (dtype) {
        case K1_DTYPE_BF16:
            return launch_backward<__nv_bfloat16>(fn, logits, L, D, col_offset, targets, lse,
                                                  entropy, g_logp, g_ent, g_lse, d_logits, s);
        case K1_DTYPE_F16:
            return launch_backward<__half>(fn, logits, L, D, col_offset, targets, lse, entropy,
                                           g_logp, g_ent, g_lse, d_logits, s);
        default:
            return launch_backward<float>(fn, logits, L, D, col_offset, targets, lse, entropy,
                                          g_logp, g_ent, g_lse, d_logits, s);
    }
}

int k1_fused_logprob_entropy_v1_backward(
    const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t inner_rows,
    int64_t inner_stride, int64_t outer_stride, const int64_t* targets, const float* lse,
    const float* entropy, const float* g_logp, const float* g_ent, const float* g_lse,
    void* d_logits, int64_t d_inner_stride, int64_t d_outer_stride, void* stream) {
    return backward_impl("k1_fused_logprob_entropy_v1_backward", logits, dtype, n_rows, vocab,
                         inner_rows, inner_stride, outer_stride, 0, targets, lse, entropy,
                         g_logp, g_ent, g_lse, d_logits, d_inner_stride, d_outer_stride, stream);
}

int k1_fused_logprob_entropy_scaled(const void* logits, int dtype, int64_t n_rows,
                                    int64_t vocab, int64_t inner_rows, int64_t inner_stride,
                                    int64_t outer_stride, float scale, const int64_t* targets,
                                    float* logprob, float* entropy, float* lse, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    static const char* fn = "k1_fused_logprob_entropy_scaled";
    Rows L{n_rows, vocab, inner_rows, inner_stride, outer_stride};
    int rc = check_common(fn, logits, dtype, L);
    if (rc) return rc;
    rc = check_scale(fn, scale);
    if (rc) return rc;
    if (n_rows == 0) return K1_OK;
    if (!targets || !logprob || !entropy || !lse)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets or output pointer", fn);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (scale == 1.f)  // x * 1 rounds to x: the unscaled kernel gives the same bits
        return k1_fused_logprob_entropy_v1(logits, dtype, n_rows, vocab, inner_rows, inner_stride,
                                           outer_stride, targets, logprob, entropy, lse,
                                           workspace, workspace_bytes, stream);
    switch (dtype) {
        case K1_DTYPE_BF16:
            return launch_forward<__nv_bfloat16, false, true>(fn, logits, L, 0, targets, logprob,
                                                              entropy, lse, nullptr, workspace,
                                                              workspace_bytes, s, scale);
        case K1_DTYPE_F16:
            return launch_forward<__half, false, true>(fn, logits, L, 0, targets, logprob, entropy,
                                                       lse, nullptr, workspace, workspace_bytes, s,
                                                       scale);
        default:
            return launch_forward<float, false, true>(fn, logits, L, 0, targets, logprob, entropy,
                                                      lse, nullptr, workspace, workspace_bytes, s,
                                                      scale);
    }
}

int k1_fused_logprob_entropy_scaled_backward(
    const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t inner_rows,
    int64_t inner_stride, int64_t outer_stride, float scale, const int64_t* targets,
    const float* lse, const float* entropy, const float* g_logp, const float* g_ent,
    const float* g_lse, void* d_logits, int64_t d_inner_stride, int64_t d_outer_stride,
    void* stream) {
    static const char* fn = "k1_fused_logprob_entropy_scaled_backward";
    int rc = check_scale(fn, scale);
    if (rc) return rc;
    return backward_impl(fn, logits, dtype, n_rows, vocab, inner_rows, inner_stride, outer_stride,
                         0, targets, lse, entropy, g_logp, g_ent, g_lse, d_logits, d_inner_stride,
                         d_outer_stride, stream, scale);
}

int k1_vocab_shard_partials(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab,
                            int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                            int64_t vocab_offset, const int64_t* targets,
                            k1_partial* partials, void* workspace, size_t workspace_bytes,
                            void* stream) {
    static const char* fn = "k1_vocab_shard_partials";
    Rows L{n_rows, shard_vocab, inner_rows, inner_stride, outer_stride};
    int rc = check_common(fn, logits, dtype, L);
    if (rc) return rc;
    if (vocab_offset < 0) return fail(K1_ERR_INVALID_ARGUMENT, "%s: vocab_offset must be >= 0", fn);
    if (n_rows == 0) return K1_OK;
    if (!targets || !partials)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets or partials", fn);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (dtype) {
        case K1_DTYPE_BF16:
            return launch_forward<__nv_bfloat16, true>(fn, logits, L, vocab_offset, targets,
                                                       nullptr, nullptr, nullptr, partials,
                                                       workspace, workspace_bytes, s);
        case K1_DTYPE_F16:
            return launch_forward<__half, true>(fn, logits, L, vocab_offset, targets, nullptr,
                                                nullptr, nullptr, partials, workspace,
                                                workspace_bytes, s);
        default:
            return launch_forward<float, true>(fn, logits, L, vocab_offset, targets, nullptr,
                                               nullptr, nullptr, partials, workspace,
                                               workspace_bytes, s);
    }
}

int k1_vocab_combine(const k1_partial* gathered, int n_shards, int64_t n_rows, float* logprob,
                     float* entropy, float* lse, void* stream) {
    static const char* fn = "k1_vocab_combine";
    if (n_shards < 1) return fail(K1_ERR_INVALID_ARGUMENT, "%s: n_shards must be >= 1", fn);
    if (n_rows < 0) return fail(K1_ERR_INVALID_ARGUMENT, "%s: n_rows must be >= 0", fn);
    if (n_rows == 0) return K1_OK;
    if (!gathered || !logprob || !entropy || !lse)
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL pointer argument", fn);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int threads = 128;
    const int64_t blocks = (n_rows + threads - 1) / threads;
    launch(k1::k1_vocab_combine_kernel, blocks, threads, 0, s, gathered, n_shards, n_rows,
           logprob, entropy, lse);
    return check_launch(fn);
}

int k1_vocab_shard_scaled_backward(const void* logits, int dtype, int64_t n_rows,
                                   int64_t shard_vocab, int64_t inner_rows, int64_t inner_stride,
                                   int64_t outer_stride, int64_t vocab_offset, float scale,
                                   const int64_t* targets, const float* lse, const float* entropy,
                                   const float* g_logp, const float* g_ent, const float* g_lse,
                                   void* d_logits, int64_t d_inner_stride, int64_t d_outer_stride,
                                   void* stream) {
    static const char* fn = "k1_vocab_shard_scaled_backward";
    int rc = check_scale(fn, scale);
    if (rc) return rc;
    if (vocab_offset < 0) return fail(K1_ERR_INVALID_ARGUMENT, "%s: vocab_offset must be >= 0", fn);
    return backward_impl(fn, logits, dtype, n_rows, shard_vocab, inner_rows, inner_stride,
                         outer_stride, vocab_offset, targets, lse, entropy, g_logp, g_ent, g_lse,
                         d_logits, d_inner_stride, d_outer_stride, stream, scale);
}

int k1_vocab_shard_backward(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab,
                            int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                            int64_t vocab_offset, const int64_t* targets, const float* lse,
                            const float* entropy, const float* g_logp, const float* g_ent,
                            const float* g_lse, void* d_logits, int64_t d_inner_stride,
                            int64_t d_outer_stride, void* stream) {
    if (vocab_offset < 0)
        return fail(K1_ERR_INVALID_ARGUMENT, "k1_vocab_shard_backward: vocab_offset must be >= 0");
    return backward_impl("k1_vocab_shard_backward", logits, dtype, n_rows, shard_vocab,
                         inner_rows, inner_stride, outer_stride, vocab_offset, targets, lse,
                         entropy, g_logp, g_ent, g_lse, d_logits, d_inner_stride,
                         d_outer_stride, stream);
}


size_t k1_lm_head_workspace_bytes(int64_t n_rows, int64_t hidden_dim, int64_t vocab, int device) {
    if (n_rows < 1 || vocab < 1 || hidden_dim < 1 || device < 0 || device >= kMaxDevices) return 0;
    LmhShape sh;
    if (lmh_shape(n_rows, hidden_dim, vocab, device, &sh) != K1_OK) return 0;
    return lmh_workspace_bytes(n_rows, sh);
}

int k1_lm_head_forward(const void* hidden, const void* weight, int64_t n_rows, int64_t hidden_dim,
                       int64_t vocab, float scale, const int64_t* targets, float* logprob,
                       float* entropy, float* lse, void* logits_out, int64_t logits_stride,
                       void* workspace, size_t workspace_bytes, void* stream) {
    static const char* fn = "k1_lm_head_forward";
    if (n_rows > 0 && (!logprob || !entropy || !lse))
        return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL targets or output pointer", fn);
    return lmh_forward(fn, hidden, weight, n_rows, hidden_dim, vocab, 0, scale, targets, logprob,
                       entropy, lse, nullptr, logits_out, logits_stride, workspace, workspace_bytes,
                       stream);
}

int k1_lm_head_shard_partials(const void* hidden, const void* weight_shard, int64_t n_rows,
                              int64_t hidden_dim, int64_t shard_vocab, int64_t vocab_offset,
                              float scale, const int64_t* targets, k1_partial* partials,
                              void* logits_out, int64_t logits_stride, void* workspace,
                              size_t workspace_bytes, void* stream) {
    static const char* fn = "k1_lm_head_shard_partials";
    if (vocab_offset < 0) return fail(K1_ERR_INVALID_ARGUMENT, "%s: vocab_offset must be >= 0", fn);
    if (n_rows > 0 && !partials) return fail(K1_ERR_INVALID_ARGUMENT, "%s: NULL partials", fn);
    return lmh_forward(fn, hidden, weight_shard, n_rows, hidden_dim, shard_vocab, vocab_offset, scale,
                       targets, nullptr, nullptr, nullptr, partials, logits_out, logits_stride,
                       workspace, workspace_bytes, stream);
}

int k1_lm_head_backward(const void* hidden, const void* weight, int64_t n_rows, int64_t hidden_dim,
                        int64_t vocab, float scale, const int64_t* targets, const float* lse,
                        const float* entropy, const float* g_logp, const float* g_ent,
                        const float* g_lse, void* d_logits, int64_t d_stride, void* stream) {
    return lmh_backward("k1_lm_head_backward", hidden, weight, n_rows, hidden_dim, vocab, 0, scale,
                        targets, lse, entropy, g_logp, g_ent, g_lse, d_logits, d_stride, stream);
}

int k1_lm_head_shard_backward(const void* hidden, const void* weight_shard, int64_t n_rows,
                              int64_t hidden_dim, int64_t shard_vocab, int64_t vocab_offset,
                              float scale, const int64_t* targets, const float* lse,
                              const float* entropy, const float* g_logp, const float* g_ent,
                              const float* g_lse, void* d_logits, int64_t d_stride, void* stream) {
    static const char* fn = "k1_lm_head_shard_backward";
    if (vocab_offset < 0) return fail(K1_ERR_INVALID_ARGUMENT, "%s: vocab_offset must be >= 0", fn);
    return lmh_backward(fn, hidden, weight_shard, n_rows, hidden_dim, shard_vocab, vocab_offset,
                        scale, targets, lse, entropy, g_logp, g_ent, g_lse, d_logits, d_stride,
                        stream);
}

#ifdef K1_WAIT_TEST
// Only in the wait-timeout test library (built with -DK1_WAIT_TEST and short wait limits;
// not part of libk1_b200.so): sets the knobs that make one block's bounded waits run out
// on the current device.  withhold: the backward ring's block 0, and the LM head's CTA 0,
// issue no bulk copy from that copy number on; skip_grab: the one-block-per-SM forward's
// block 0 drops that grab.  -1 turns a knob off.
int k1_test_set_knobs(long long withhold, long long skip_grab) {
    cudaError_t e = cudaMemcpyToSymbol(k1::k1_test_withhold, &withhold, sizeof withhold);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(k1::k1_test_skip_grab, &skip_grab, sizeof skip_grab);
    if (e != cudaSuccess) return fail(K1_ERR_CUDA, "k1_test_set_knobs: %s", cudaGetErrorString(e));
    return K1_OK;
}
#endif

}  // extern "C"
