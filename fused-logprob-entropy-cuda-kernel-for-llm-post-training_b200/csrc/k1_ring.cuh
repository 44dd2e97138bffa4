// k1_ring.cuh -- bulk-copy (TMA) ring variants of the forward and backward kernels.
//
// One producer warp per block streams the block's rows in chunks of up to SBYTES with
// cp.async.bulk (global -> shared, completion counted on an mbarrier) into a ring of
// STAGES buffers; NCW consumer warps reduce (forward) or transform and store (backward)
// straight out of shared memory, then release the buffer on a second mbarrier.  The
// number of bytes in flight per SM is set by the ring size, not by registers.
//
// Every mbarrier wait is bounded (kMaxTries polls with a suspend hint, a few seconds in
// all).  A wait that runs out sets the device word k1_ring_error and the thread stops
// waiting; the producer drains every copy it issued before it exits.  No wait depends
// on another block or another GPU.  Bulk copies are plain global -> shared copies of this
// GPU's memory into this block's own shared memory; source and size are multiples of 16
// bytes on the vector path.
#pragma once

#include "k1_kernels.cuh"

#ifndef K1_RING_MINB
#define K1_RING_MINB 1
#endif
#ifndef K1_RING_FWD_MINB
#define K1_RING_FWD_MINB 1
#endif
// 1: the backward's producer issues its first STAGES bulk copies before waiting for the
// previous kernel of the stream (programmatic dependent launch), so they overlap that
// kernel's tail.  That read of the logits is only correct when the previous kernel does
// not write them, which the library cannot know: a GEMM that produced the logits right
// before the backward (an LM head) may trigger its dependents before its last stores,
// and only griddepcontrol.wait makes a primary's writes visible.  The gain was under 1 %
// of a step, so every build waits before its first copy (0).
#ifndef K1_RING_EARLY
#define K1_RING_EARLY 0
#endif

// Polls of a bounded mbarrier wait before it gives up (each poll suspends for at most
// kSuspendHintNs).  The wait-timeout test library is built with a small value.
#ifndef K1_RING_MAX_TRIES
#define K1_RING_MAX_TRIES 4096
#endif

namespace k1 {

__device__ unsigned k1_ring_error;

#ifdef K1_WAIT_TEST
// Test-only knob (compiled into the wait-timeout test library only): block 0's producer
// issues no copy from its chunk number k1_test_withhold on, so the consumers' waits for
// that chunk run out.  -1: off.
__device__ long long k1_test_withhold = -1;
#endif

namespace ring {

constexpr int kMaxTries = K1_RING_MAX_TRIES;  // x up to 1 ms suspend hint per poll
constexpr uint32_t kSuspendHintNs = 1000000;

__device__ __forceinline__ uint32_t saddr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void arrive_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of parity `parity`; false (and the error word set) if it
// did not complete in time.
__device__ __forceinline__ bool wait(uint64_t* b, uint32_t parity) {
    for (int i = 0; i < kMaxTries; ++i)
        if (try_wait(b, parity)) return true;
    atomicOr(&k1_ring_error, 1u);
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(saddr(dst)),
        "l"(src), "r"(bytes), "r"(saddr(bar))
        : "memory");
}

// The chunk sequence of one block: its flattened vector range [start, end) walked row by
// row, each row segment cut into chunks of at most SV vectors.  Producer and consumers
// walk the same sequence.
struct ChunkWalk {
    int64_t pos, end, r, j0, j1;
    __device__ __forceinline__ void begin(int64_t start, int64_t stop, int64_t vpr) {
        pos = start;
        end = stop;
        r = start / vpr;
        j0 = start - r * vpr;
        j1 = min(vpr, j0 + (end - pos));
    }
    __device__ __forceinline__ void next_row(int64_t vpr) {
        pos += j1 - j0;
        ++r;
        j0 = 0;
        j1 = min(vpr, end - pos);
    }
};

// Producer: issue every chunk of the block, SBYTES at most each, into the ring.  With
// PEEL the units are elements and each row segment contributes only its 16-byte aligned
// interior (see peel); otherwise units are whole vectors.
// EARLY: the first STAGES copies go out before this thread waits for the previous kernel
// of the stream (pdl_wait); otherwise the caller has waited already.
template <typename T, bool PEEL, int STAGES, int SV, bool EARLY = false>
__device__ __forceinline__ void produce(const void* base, const RowLayout& lay, int64_t vpr,
                                        int64_t start, int64_t end, uint4* ring, uint64_t* full,
                                        uint64_t* empty) {
    ChunkWalk w;
    w.begin(start, end, vpr);
    uint32_t k = 0;
    bool ok = true;
    bool waited = !EARLY;
    while (ok && w.pos < w.end) {
        const T* rowp = reinterpret_cast<const T*>(base) + lay.offset(w.r);
        const uint4* src;
        int64_t c0, c1;  // the segment's vectors, relative to src
        if constexpr (PEEL) {
            int64_t a0, a1;
            peel(rowp, w.j0, w.j1, a0, a1);
            src = reinterpret_cast<const uint4*>(rowp + a0);
            c0 = 0;
            c1 = (a1 - a0) / DT<T>::kEPV;
        } else {
            src = reinterpret_cast<const uint4*>(rowp);
            c0 = w.j0;
            c1 = w.j1;
        }
        for (int64_t jj = c0; jj < c1; jj += SV) {
            const uint32_t n = (uint32_t)min((int64_t)SV, c1 - jj);
            const uint32_t s = k % STAGES, use = k / STAGES;
            if (!waited && k == (uint32_t)STAGES) {
                pdl_wait();
                waited = true;
            }
            if (use > 0 && !wait(&empty[s], (use - 1) & 1)) {
                ok = false;
                break;
            }
#ifdef K1_WAIT_TEST
            if (blockIdx.x == 0 && (long long)k == k1_test_withhold) {
                ok = false;
                break;
            }
#endif
            arrive_expect(&full[s], n * 16u);
            bulk_g2s(ring + (size_t)s * SV, src + jj, n * 16u, &full[s]);
            ++k;
        }
        w.next_row(vpr);
    }
    if (!waited) pdl_wait();
    // drain: every issued copy has landed before this thread returns
    for (uint32_t i = (k > (uint32_t)STAGES ? k - STAGES : 0u); i < k; ++i)
        wait(&full[i % STAGES], (i / STAGES) & 1);
}

}  // namespace ring

template <typename T, int NCW, int STAGES, int SBYTES, bool SHARD>
__global__ void __launch_bounds__((NCW + 1) * 32, K1_RING_FWD_MINB) k1_fwd_ring_kernel(FwdParams p) {
    constexpr int NC = NCW * 32;
    constexpr int BAR = 1;  // named barrier of the consumer warps (the producer returns early)
    constexpr int SV = SBYTES / 16;
    constexpr int VPT = SV / NC;
    static_assert(SV % NC == 0, "stage must hold a whole number of vectors per consumer");
    extern __shared__ __align__(128) uint4 ring_buf[];
    __shared__ __align__(8) uint64_t full[STAGES];
    __shared__ __align__(8) uint64_t empty[STAGES];
    __shared__ FwdSmem<NC> sm;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ring::bar_init(&full[s], 1);
            ring::bar_init(&empty[s], NCW);
        }
        ring::fence_init();
    }
    __syncthreads();
    const int64_t G = gridDim.x, b = blockIdx.x;
    const int64_t start = piece_start(b, p.total, G), end = piece_start(b + 1, p.total, G);
    if (warp == NCW) {
        if (lane == 0)
            ring::produce<T, false, STAGES, SV>(p.logits, p.lay, p.vpr, start, end, ring_buf,
                                                full, empty);
        return;
    }
    const int tid = threadIdx.x;
    const uint32_t pw = DT<T>::kPadWord;
    ring::ChunkWalk w;
    w.begin(start, end, p.vpr);
    const int64_t first_row = w.r;
    int64_t split_row[2] = {-1, -1};
    unsigned split_prev[2] = {0u, 0u};
    int count = 0, buf = 0;
    uint32_t k = 0;
    bool ok = true;
    while (w.pos < w.end) {
        const int64_t r = w.r, j0 = w.j0, j1 = w.j1;
        const T* rowp = reinterpret_cast<const T*>(p.logits) + p.lay.offset(r);
        FwdState st;
        st.init();
        for (int64_t jj = j0; jj < j1; jj += SV) {
            const int64_t n = min((int64_t)SV, j1 - jj);
            const uint32_t s = k % STAGES, use = k / STAGES;
            if (ok) ok = ring::wait(&full[s], use & 1);
            const uint4* stage = ring_buf + (size_t)s * SV;
            if (ok) {
                uint4 v[VPT];
#pragma unroll
                for (int u = 0; u < VPT; ++u)
                    v[u] = (tid + u * NC < n) ? stage[tid + u * NC] : make_uint4(pw, pw, pw, pw);
                fwd_chunk<T, VPT>(v, st, false);
            }
            __syncwarp();
            if (lane == 0) ring::arrive(&empty[s]);
            ++k;
        }
        RowPartial part;
        if (!seg_merge<NC, BAR>(st.m, st.z64(), st.t64(), st.m <= DT<T>::kLowest,
                                st.saw_neg_inf(), sm, buf, part)) {
            // rare: the segment holds -inf logits; stream it again from global, clamped
            st.init();
            fwd_stream_vec<T, false, NC, 4>(rowp, j0, j1, st, tid, true, 1.f);
            seg_merge<NC, BAR>(st.m, st.z64(), st.t64(), st.m <= DT<T>::kLowest, false, sm, buf,
                               part);
        }
        buf ^= 1;
        if (j0 == 0 && j1 == p.vpr) {
            if (tid == 0) {
                sm.done_row[count] = r;
                sm.done_part[count] = part;
            }
            if (++count == kRowCap) {
                fwd_flush_rows<T, NC, BAR, SHARD>(p, sm, count);
                count = 0;
            }
        } else {
            const int slot = (r == first_row) ? 0 : 1;
            split_row[slot] = r;
            if (tid == 0) {
                p.ws_part[2 * b + slot] = part;
                __threadfence();
                split_prev[slot] = atomicAdd(p.ws_ticket + block_of(r * p.vpr, p.total, G), 1u);
            }
        }
        w.next_row(p.vpr);
    }
    if (tid == 0) {
        sm.split_prev[0] = split_prev[0];
        sm.split_prev[1] = split_prev[1];
    }
    fwd_flush_rows<T, NC, BAR, SHARD>(p, sm, count);
    const int slot = tid >> 5;
    if (slot < 2) {
        const int64_t sr = slot == 0 ? split_row[0] : split_row[1];
        if (sr >= 0) {
            const int64_t bf = block_of(sr * p.vpr, p.total, G);
            const int64_t bl = block_of((sr + 1) * p.vpr - 1, p.total, G);
            const unsigned prev = slot == 0 ? sm.split_prev[0] : sm.split_prev[1];
            if (prev == (unsigned)(bl - bf)) fwd_merge_split_row<T, SHARD>(p, sr);
        }
    }
}

// PEEL: rows that are not whole vectors (units are elements); the logits and gradient rows
// must share their 16-byte misalignment (checked by the launcher).  Each row segment's
// aligned interior goes through the ring, its head and tail elements are handled by the
// consumer threads directly.
template <typename T, int NCW, int STAGES, int SBYTES, bool SCALED = false, bool PEEL = false>
__global__ void __launch_bounds__((NCW + 1) * 32, K1_RING_MINB) k1_bwd_ring_kernel(BwdParams p) {
    using D = DT<T>;
    constexpr int NC = NCW * 32;
    constexpr int SV = SBYTES / 16;
    constexpr int VPT = SV / NC;
    constexpr int EPV = D::kEPV;
    static_assert(SV % NC == 0, "stage must hold a whole number of vectors per consumer");
    extern __shared__ __align__(128) uint4 ring_buf[];
    __shared__ __align__(8) uint64_t full[STAGES];
    __shared__ __align__(8) uint64_t empty[STAGES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (!K1_RING_EARLY) pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ring::bar_init(&full[s], 1);
            ring::bar_init(&empty[s], NCW);
        }
        ring::fence_init();
    }
    __syncthreads();
    const int64_t G = gridDim.x, b = blockIdx.x;
    const int64_t start = b * p.total / G, end = (b + 1) * p.total / G;
    if (warp == NCW) {
        if (lane == 0)
            ring::produce<T, PEEL, STAGES, SV, K1_RING_EARLY != 0>(p.logits, p.lay, p.vpr, start,
                                                                  end, ring_buf, full, empty);
        return;
    }
    if (K1_RING_EARLY) pdl_wait();  // the consumers read the forward's outputs
    const int tid = threadIdx.x;
    ring::ChunkWalk w;
    w.begin(start, end, p.vpr);
    uint32_t k = 0;
    bool ok = true;
    while (w.pos < w.end) {
        const int64_t r = w.r;
        const T* xr = reinterpret_cast<const T*>(p.logits) + p.lay.offset(r);
        T* dr = reinterpret_cast<T*>(p.dlogits) + p.dlay.offset(r);
        BwdRow q;
        q.lse = p.lse[r];
        q.ent = p.entropy[r];
        q.gl = p.g_logp ? p.g_logp[r] : 0.f;
        q.ge = p.g_ent ? p.g_ent[r] : 0.f;
        q.gs = p.g_lse ? p.g_lse[r] : 0.f;
        q.c0 = q.gs - q.gl - q.ge * q.ent;
        {
            const int64_t tg = p.targets[r];
            const int64_t tl = tg - p.col_offset;
            q.tl = (tg >= 0 && tl >= 0 && tl < p.vocab) ? tl : -1;
        }
        // the segment's vectors [c0, c1) relative to the vector base dv (the producer's
        // chunks); tl_rel = target column relative to dv's first element
        uint4* dv;
        int64_t c0, c1, tl_rel;
        if constexpr (PEEL) {
            int64_t a0, a1;
            peel(xr, w.j0, w.j1, a0, a1);
            dv = reinterpret_cast<uint4*>(dr + a0);
            c0 = 0;
            c1 = (a1 - a0) / EPV;
            tl_rel = q.tl - a0;
            const int64_t nh = a0 - w.j0, ne = nh + (w.j1 - a1);  // at most 2 (EPV - 1)
            if (tid < ne)
                bwd_element<T, SCALED>(xr, dr, tid < nh ? w.j0 + tid : a1 + (tid - nh), q,
                                       p.scale);
        } else {
            dv = reinterpret_cast<uint4*>(dr);
            c0 = w.j0;
            c1 = w.j1;
            tl_rel = q.tl;
        }
        for (int64_t jj = c0; jj < c1; jj += SV) {
            const int64_t n = min((int64_t)SV, c1 - jj);
            const uint32_t s = k % STAGES, use = k / STAGES;
            if (ok) ok = ring::wait(&full[s], use & 1);
            const uint4* stage = ring_buf + (size_t)s * SV;
            if (ok) {
#pragma unroll
                for (int u = 0; u < VPT; ++u) {
                    const int64_t i = tid + u * NC;
                    if (i < n) {
                        const int64_t jv = jj + i;
                        uint4 o = bwd_vector<T, SCALED>(stage[i], q, p.scale);
                        const uint64_t kk = (uint64_t)(tl_rel - jv * EPV);
                        if (kk < (uint64_t)EPV)
                            o = vec_set<T>(o, (int)kk, bwd_target_out<T>(xr, q, p.scale));
                        stg_stream(dv + jv, o);
                    }
                }
            } else {
                // a wait ran out (k1_ring_error is set): this thread's share of every
                // remaining chunk becomes NaN, so the failure shows in the gradient
                // without the host reading the error word
                const uint32_t nw = DT<T>::kNaNWord;
#pragma unroll
                for (int u = 0; u < VPT; ++u) {
                    const int64_t i = tid + u * NC;
                    if (i < n) stg_stream(dv + jj + i, make_uint4(nw, nw, nw, nw));
                }
            }
            __syncwarp();
            if (lane == 0) ring::arrive(&empty[s]);
            ++k;
        }
        w.next_row(p.vpr);
    }
}

}  // namespace k1
