// k1_fwd_sm.cuh -- forward for a few wide rows per SM: one block per SM streams its rows
// as a sequence of fixed pieces ("grabs") that its warps take in turn, and rows are merged
// without barriers.
//
// With a few rows per SM (1024 rows of 152 064 logits on 148 SMs: 6.9 per SM), a queue
// of whole rows for several row groups per SM drains badly (the last round of rows runs
// on a fraction of the groups), and splitting rows between blocks costs block-wide merges
// and published partials.  Here block b owns rows b, b + G, b + 2G, ... (G = grid).  Each
// row is cut into `gpr` grabs of GC chunks of 32 x U vectors; the block's warps take the
// grabs of its rows in order from a shared-memory counter, so a warp that runs slower
// (the schedulers do not serve warps equally) simply takes fewer of them.  A warp reduces
// its grab from a fresh state, parks its lanes' states (m, z, t) in the row's slot and
// counts the grab in; the warp that completes the row's count merges the parked states in
// grab order and writes the row's outputs.  A grab's states depend only on its logits and
// the merge order is fixed, so results do not depend on which warp took which grab.
// 16 warps of 128 registers each keep the next chunk's loads in flight while a chunk is
// reduced (two register buffers), so a warp does not idle between chunks; grabs are at
// least 8 chunks (32 KB) long, which keeps the per-grab park and count to a few percent.
//
// -inf logits: a lane whose fast (unclamped) reduction of a grab turned t into NaN reduces
// the grab again with every logit clamped to the lowest finite value; clamping changes
// nothing else, so this equals a clamped pass over the whole row.
//
// Row slots: R slots are reused round robin; a warp parking a grab of row j waits until
// row j - R has been merged (its grabs were handed out at least R - 1 rows earlier, so
// this wait is normally already over).  Every wait depends only on warps of the same
// block holding grabs of earlier rows, so it always ends; it is still bounded (polls with
// a suspend hint) and sets bit 2 of k1_ring_error instead of hanging, and the two rows it
// leaves unfinished get NaN outputs.
#pragma once

#include "k1_ring.cuh"

#ifndef K1_SM_SLOTS
#define K1_SM_SLOTS 4
#endif
#ifndef K1_SM_MAX_GRABS
#define K1_SM_MAX_GRABS 32  // grabs per row at most (larger rows get larger grabs)
#endif
#ifndef K1_SM_PREFETCH
#define K1_SM_PREFETCH 1  // next chunk's loads in flight while a chunk is reduced
#endif
#ifndef K1_SM_GRAB_CHUNKS
#define K1_SM_GRAB_CHUNKS 8  // chunks of 32 x U vectors per grab at least
#endif

namespace k1 {

struct SmFwdSmem {
    static constexpr int R = K1_SM_SLOTS;
    static constexpr int GM = K1_SM_MAX_GRABS;
    double z[R][GM][32];
    double t[R][GM][32];
    float m[R][GM][32];  // -inf: the lane saw no logit of the grab
    float xt[R];         // the row's target logit, written by the warp whose grab holds it
    int slot_row[R];     // block-local row that slot s accepts
    int done[R];         // grabs of that row parked so far
    int next;            // next grab of the block's sequence
};

// Polls of a row-slot wait before it gives up (each poll sleeps about 64 ns or more).
// The wait-timeout test library is built with a small value.
#ifndef K1_SM_MAX_POLLS
#define K1_SM_MAX_POLLS (1 << 22)
#endif
constexpr int kSmMaxPolls = K1_SM_MAX_POLLS;

#ifdef K1_WAIT_TEST
// Test-only knob (compiled into the wait-timeout test library only): block 0 drops its
// grab number k1_test_skip_grab instead of parking it, so that row never completes and
// the row that next needs its slot waits until the wait runs out.  -1: off.
__device__ long long k1_test_skip_grab = -1;
#endif

// Grab geometry of a row of `cpr` chunks: chunks per grab and grabs per row.
__device__ __forceinline__ void sm_grabs(int64_t cpr, int& gc, int& gpr) {
    int64_t c = (cpr + SmFwdSmem::GM - 1) / SmFwdSmem::GM;
    if (c < K1_SM_GRAB_CHUNKS) c = K1_SM_GRAB_CHUNKS;
    gc = (int)c;
    gpr = (int)((cpr + c - 1) / c);
}

// Park a warp's grab g of block-local row j, in two steps: sm_store waits for the row's
// slot and stores the lanes' states (and the target logit when the grab holds it);
// sm_count counts the grab in and returns true for the warp that completed the row, which
// must then call sm_merge.  Returns false from sm_store when the slot wait ran out.
template <typename T>
__device__ __forceinline__ bool sm_store(SmFwdSmem& sm, int j, int g, const FwdState& st,
                                         bool cap, float xt, int lane) {
    const int s = j % SmFwdSmem::R;
    int ok = 1;
    if (lane == 0) {
        volatile int* sr = &sm.slot_row[s];
        int n = 0;
        while (*sr != j) {
            if (++n > kSmMaxPolls) {
                atomicOr(&k1_ring_error, 4u);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
    const bool empty = st.m <= DT<T>::kLowest;
    sm.m[s][g][lane] = empty ? -INFINITY : st.m;
    sm.z[s][g][lane] = st.z64();
    sm.t[s][g][lane] = st.t64();
    if (cap && lane == 0) sm.xt[s] = xt;
    return true;
}

__device__ __forceinline__ bool sm_count(SmFwdSmem& sm, int j, int gpr, int lane) {
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&sm.done[j % SmFwdSmem::R], 1) == gpr - 1;
    }
    return __shfl_sync(0xffffffffu, last, 0) != 0;
}

// Merge the parked states of row j (global row r) in grab order, write its outputs and
// hand the slot to row j + R.
template <bool SHARD>
__device__ __forceinline__ void sm_merge(const FwdParams& p, SmFwdSmem& sm, int j, int gpr,
                                         int64_t r, bool has, int lane) {
    constexpr int R = SmFwdSmem::R;
    const int s = j % R;
    __threadfence_block();
    float M = -INFINITY;
    for (int i = 0; i < gpr; ++i) M = fmax_nan(M, sm.m[s][i][lane]);
    M = warp_max_nan(M);
    double zc = 0.0, tc = 0.0;
    for (int i = 0; i < gpr; ++i) {
        const float mi = sm.m[s][i][lane];
        if (mi != -INFINITY) {
            const float dm = mi - M;
            const float sc = (dm == 0.f) ? 1.f : ex2(dm * kLog2e);
            const double z = sm.z[s][i][lane];
            zc += (double)sc * z;
            tc += (double)sc * (sm.t[s][i][lane] + (double)dm * z);
        }
    }
    zc = warp_sum(zc);
    tc = warp_sum(tc);
    if (lane == 0) {
        RowPartial part;
        part.z = zc;
        part.t = tc;
        part.m = M;
        part.pad = 0.f;
        if (M == -INFINITY) part.z = part.t = 0.0;
        const float x = has ? sm.xt[s] : 0.f;
        if constexpr (SHARD) {
            k1_partial o;
            o.z = part.z;
            o.t = part.t;
            o.m = part.m;
            o.x_t = x;
            o.has_target = has ? 1 : 0;
            o.reserved = 0;
            p.partials[r] = o;
        } else {
            finalize_row(part, has ? (double)x : 0.0, p.logprob + r, p.entropy + r, p.lse + r);
        }
        sm.done[s] = 0;
        __threadfence_block();
        *(volatile int*)&sm.slot_row[s] = j + R;
    }
}

// A slot wait ran out (k1_ring_error bit 2 is set): the warp could not park its grab of
// block-local row j, and the row still holding the slot can no longer complete either.
// Both rows' outputs become NaN, so the failure shows without the host reading the
// error word.
template <bool SHARD>
__device__ __forceinline__ void sm_fail(const FwdParams& p, const SmFwdSmem& sm, int j, int lane) {
    if (lane != 0) return;
    const float nan = __int_as_float(0x7fc00000);
    const int jo = *(volatile const int*)&sm.slot_row[j % SmFwdSmem::R];
    const int64_t rows[2] = {blockIdx.x + (int64_t)j * gridDim.x,
                             (jo >= 0 && jo < j) ? blockIdx.x + (int64_t)jo * gridDim.x : -1};
    for (int i = 0; i < 2; ++i) {
        const int64_t r = rows[i];
        if (r < 0 || r >= p.n_rows) continue;
        if constexpr (SHARD) {
            k1_partial o;
            o.z = o.t = (double)nan;
            o.m = nan;
            o.x_t = nan;
            o.has_target = 0;
            o.reserved = 0;
            p.partials[r] = o;
        } else {
            p.logprob[r] = nan;
            p.entropy[r] = nan;
            p.lse[r] = nan;
        }
    }
}

// Element offset of row r; 32-bit division when the operands fit (the common case).
__device__ __forceinline__ int64_t sm_row_offset(const RowLayout& lay, int64_t r) {
    if (lay.inner_rows == 1) return r * lay.outer_stride;
    int64_t o;
    if (r < 0x7fffffff && lay.inner_rows < 0x7fffffff)
        o = (int64_t)((unsigned)r / (unsigned)lay.inner_rows);
    else
        o = r / lay.inner_rows;
    return o * lay.outer_stride + (r - o * lay.inner_rows) * lay.inner_stride;
}

// One block of NW warps per SM (launch with gridDim.x <= n_rows, rows of fewer than 2^31
// vectors and sizeof(SmFwdSmem) bytes of dynamic shared memory); vector path only.
template <typename T, int NW, int U, bool SHARD, bool SCALED, bool PF>
__global__ void __launch_bounds__(NW * 32, 1) k1_fwd_sm_kernel(FwdParams p) {
    extern __shared__ __align__(16) unsigned char k1_sm_raw[];
    SmFwdSmem& sm = *reinterpret_cast<SmFwdSmem*>(k1_sm_raw);
    constexpr int CV = 32 * U;  // vectors per chunk
    constexpr int EPV = DT<T>::kEPV;
    if (threadIdx.x < SmFwdSmem::R) {
        sm.slot_row[threadIdx.x] = threadIdx.x;
        sm.done[threadIdx.x] = 0;
    }
    if (threadIdx.x == 0) sm.next = NW;
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x, G = gridDim.x;
    if (b >= p.n_rows) return;
    const int nrb = (int)((p.n_rows - 1 - b) / G + 1);
    const int vpr = (int)p.vpr;
    int gc, gpr;
    sm_grabs((vpr + CV - 1) / CV, gc, gpr);
    const int total = nrb * gpr;
    const int gv = gc * CV;  // vectors per grab
    int k = threadIdx.x >> 5;  // the first NW grabs go to the warps in order
    while (k < total) {
        int kn = 0;
        if (lane == 0) kn = atomicAdd(&sm.next, 1);  // the grab after this one
        const int j = (int)((unsigned)k / (unsigned)gpr), g = k - j * gpr;
        const int64_t r = b + (int64_t)j * G;
        const T* rowp = reinterpret_cast<const T*>(p.logits) + sm_row_offset(p.lay, r);
        const int64_t tg = p.targets[r];
        const int a = g * gv, e = min(vpr, a + gv);
        FwdState st;
        st.init();
        fwd_stream_vec<T, SCALED, 32, U, PF>(rowp, a, e, st, lane, false, p.scale);
        if (st.saw_neg_inf()) {
            st.init();
            fwd_stream_vec<T, SCALED, 32, U, false>(rowp, a, e, st, lane, true, p.scale);
        }
        const int64_t tt = SHARD ? tg - p.col_offset : tg;
        const bool has = tg >= 0 && tt >= 0 && tt < p.vocab;
        bool cap = false;
        float xt = 0.f;
        if (has && tt / EPV >= a && tt / EPV < e) {
            cap = true;
            if (lane == 0) xt = target_logit<T>(rowp + tt, p.scale);
        }
#ifdef K1_WAIT_TEST
        if (b == 0 && (long long)k == k1_test_skip_grab) {
            k = __shfl_sync(0xffffffffu, kn, 0);
            continue;
        }
#endif
        if (!sm_store<T>(sm, j, g, st, cap, xt, lane))
            sm_fail<SHARD>(p, sm, j, lane);
        else if (sm_count(sm, j, gpr, lane))
            sm_merge<SHARD>(p, sm, j, gpr, r, has, lane);
        k = __shfl_sync(0xffffffffu, kn, 0);
    }
}

}  // namespace k1
