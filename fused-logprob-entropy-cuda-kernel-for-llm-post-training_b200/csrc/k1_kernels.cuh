// k1_kernels.cuh -- the K1 kernels for sm_100a.
//
// Work decomposition (forward and backward alike).  The logits are viewed as
// n_rows x vpr "units" (a unit is one 16-byte vector on the vector path, one element
// on the scalar path) and the flattened unit range [0, n_rows * vpr) is cut into
// gridDim.x equal, contiguous pieces, one per thread block.  Every block therefore
// streams the same number of bytes whatever the row count: thousands of rows give each
// block a few whole rows, a handful of rows spreads each row over many blocks
// (the split-vocab case).  A row that crosses block boundaries is finished by the
// last block to arrive at its ticket; nobody waits.
//
// The forward can also keep the last part of the range as a dynamic tail (Partition):
// fixed chunks that blocks take from an atomic counter once their own piece is done, so
// that the blocks sharing an SM (which the warp schedulers do not serve equally) finish
// together.  Chunk boundaries are fixed and a chunk is computed the same way by any
// block, so results do not depend on which block took it.
#pragma once

#include <type_traits>

#include "k1_common.cuh"
#include "../../include/k1_logprob.h"

namespace k1 {

// Block pieces: the flattened unit range [0, total) is cut into G equal contiguous pieces,
// piece b = [floor(b * total / G), floor((b + 1) * total / G)).
__device__ __forceinline__ int64_t piece_start(int64_t b, int64_t total, int64_t G) {
    return b * total / G;
}
// Block whose piece holds unit u.
__device__ __forceinline__ int64_t block_of(int64_t u, int64_t total, int64_t G) {
    return ((u + 1) * G + total - 1) / total - 1;
}

// Owners of the forward's units: G static pieces over [0, split) (piece b is block b's)
// followed by D dynamic chunks of `csize` units over [split, total) (the last one may be
// shorter), taken in order from a counter.  D = 0 (split = total) is the plain static
// split.  Every owner is non-empty (G <= split, D = ceil((total - split) / csize),
// enforced by the launcher).  start(o) is defined for 0 <= o <= G + D; start(G) = split
// comes from the static formula, and no division involves D or csize when D = 0.
struct Partition {
    int64_t total, split, G, D, csize;
    __device__ __forceinline__ int64_t start(int64_t o) const {
        return o <= G ? piece_start(o, split, G) : min(total, split + (o - G) * csize);
    }
    __device__ __forceinline__ int64_t owner_of(int64_t u) const {
        return u < split ? block_of(u, split, G) : G + (u - split) / csize;
    }
};

struct FwdParams {
    const void* logits;
    int64_t n_rows;
    int64_t vocab;
    RowLayout lay;
    int64_t vpr;         // units per row
    int64_t total;       // n_rows * vpr
    int64_t col_offset;  // global column of column 0 (vocab-parallel shards)
    const int64_t* targets;
    float* logprob;
    float* entropy;
    float* lse;
    k1_partial* partials;  // shard mode output
    RowPartial* ws_part;   // 2 slots per owner (the owner's first and last row)
    unsigned* ws_ticket;   // one counter per owner, zero between calls
    unsigned* ws_dyn;      // [next dynamic chunk, blocks done], zero between calls
    int64_t split;         // start of the dynamic tail (= total without one)
    int64_t n_dyn;         // dynamic chunks (0 = static split only)
    int64_t dyn_units;     // units per dynamic chunk
    float scale;           // logits are read as dtype(x * scale); 1 = as stored
    __device__ __forceinline__ Partition part() const {
        return Partition{total, split, (int64_t)gridDim.x, n_dyn, dyn_units};
    }
};

struct BwdParams {
    const void* logits;
    void* dlogits;
    int64_t n_rows;
    int64_t vocab;
    RowLayout lay;
    RowLayout dlay;
    int64_t vpr;
    int64_t total;
    int64_t col_offset;
    const int64_t* targets;
    const float* lse;
    const float* entropy;
    const float* g_logp;
    const float* g_ent;
    const float* g_lse;
    float scale;  // logits are read as y = dtype(x * scale), d_logits = dtype(dtype(dL/dy) * scale)
};

// ---------------------------------------------------------------------------------
// Scaled logits (sampling temperature).  The scaled entry points read every logit as
// y = dtype(x * s): the fp32 product rounded to the logits' own type, which is what an
// in-place `logits.div_(T)` leaves in the tensor (torch divides a CUDA tensor by a
// Python scalar as a multiplication by s = (float)(1.0 / T), the reciprocal taken in
// double and rounded to fp32).  Their gradient w.r.t. x is
// dtype(dtype(dL/dy) * s): the rounding of K1's own backward, then the division's
// backward.  With s = 1 both maps are the identity, so the per-row target-logit loads
// apply p.scale unconditionally; the per-element paths are compiled with and without it.
// ---------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float scale1(float x, float s) {
    return DT<T>::round1(__fmul_rn(x, s));
}

template <typename T>
__device__ __forceinline__ uint4 scale_vec(uint4 v, float s) {
    if constexpr (sizeof(T) == 2) {
        using D = DT<T>;
        return make_uint4(D::scale2(v.x, s), D::scale2(v.y, s), D::scale2(v.z, s),
                          D::scale2(v.w, s));
    } else {
        const float2 a = mul2(make_float2(__uint_as_float(v.x), __uint_as_float(v.y)), splat(s));
        const float2 b = mul2(make_float2(__uint_as_float(v.z), __uint_as_float(v.w)), splat(s));
        return make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x),
                          __float_as_uint(b.y));
    }
}

// Target logit of a row as the kernels see it (scaled like every other logit).
template <typename T>
__device__ __forceinline__ float target_logit(const T* p, float s) {
    return scale1<T>(DT<T>::load1(p), s);
}

// ---------------------------------------------------------------------------------
// Forward: per-chunk work of one thread
// ---------------------------------------------------------------------------------
// Build-time tuning knobs; the defaults are the variants measured fastest on B200.
#ifndef K1_FWD_UNROLL
#define K1_FWD_UNROLL 8
#endif
#ifndef K1_BWD_UNROLL
#define K1_BWD_UNROLL 8
#endif
#ifndef K1_FWD_MINB
#define K1_FWD_MINB 3
#endif
#ifndef K1_BWD_MINB
#define K1_BWD_MINB 3
#endif
#ifndef K1_BWD_PEEL_UNROLL
#define K1_BWD_PEEL_UNROLL 4  // vectors a thread per chunk on peeled (misaligned) rows
#endif
#ifndef K1_MIXED_ADD
#define K1_MIXED_ADD 1
#endif
#ifndef K1_FWD_PREFETCH
#define K1_FWD_PREFETCH 0
#endif

// clamp = false is the fast path: logits are used as loaded.  A -inf logit then turns t
// into NaN (0 * -inf), which the caller detects after the segment and re-streams the
// segment with clamp = true (a block-uniform flag), where every logit is first clamped
// to the lowest finite value of its type.
template <typename T, int U>
__device__ __forceinline__ void fwd_chunk(const uint4 (&v)[U], FwdState& st, bool clamp) {
    using D = DT<T>;
    if constexpr (sizeof(T) == 2) {
        uint32_t w[4 * U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            w[4 * u + 0] = v[u].x;
            w[4 * u + 1] = v[u].y;
            w[4 * u + 2] = v[u].z;
            w[4 * u + 3] = v[u].w;
        }
        if (clamp) {
#pragma unroll
            for (int i = 0; i < 4 * U; ++i) w[i] = D::clamp2(w[i]);
        }
        uint32_t mx[4 * U];
#pragma unroll
        for (int i = 0; i < 4 * U; ++i) mx[i] = w[i];
#pragma unroll
        for (int s = 2 * U; s >= 1; s >>= 1) {
#pragma unroll
            for (int i = 0; i < s; ++i) mx[i] = D::max2(mx[i], mx[i + s]);
        }
        float2 mf = D::to_f2(mx[0]);
        st.rescale(fmax_nan(mf.x, mf.y));
        const float2 nm = splat(-st.m);
#pragma unroll
        for (int i = 0; i < 4 * U; ++i) {
            if constexpr (K1_MIXED_ADD && std::is_same<T, __nv_bfloat16>::value) {
                st.accum_d(bf16x2_minus(w[i], nm.x));
            } else if constexpr (K1_MIXED_ADD && std::is_same<T, __half>::value) {
                st.accum_d(f16x2_minus(w[i], nm.x));
            } else {
                st.accum(D::to_f2(w[i]), nm);
            }
        }
        st.np += (float)(4 * U);
    } else {
        float f[4 * U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            f[4 * u + 0] = __uint_as_float(v[u].x);
            f[4 * u + 1] = __uint_as_float(v[u].y);
            f[4 * u + 2] = __uint_as_float(v[u].z);
            f[4 * u + 3] = __uint_as_float(v[u].w);
        }
        if (clamp) {
#pragma unroll
            for (int i = 0; i < 4 * U; ++i) f[i] = D::clamp1(f[i]);
        }
        float mx[4 * U];
#pragma unroll
        for (int i = 0; i < 4 * U; ++i) mx[i] = f[i];
#pragma unroll
        for (int s = 2 * U; s >= 1; s >>= 1) {
#pragma unroll
            for (int i = 0; i < s; ++i) mx[i] = fmax_nan(mx[i], mx[i + s]);
        }
        st.rescale(mx[0]);
        const float2 nm = splat(-st.m);
#pragma unroll
        for (int i = 0; i < 2 * U; ++i) st.accum(make_float2(f[2 * i], f[2 * i + 1]), nm);
        st.np += (float)(2 * U);
    }
}

template <int U, int THREADS>
__device__ __forceinline__ void load_vectors(uint4 (&v)[U], const uint4* vp, int64_t j) {
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = ldg_stream(vp + j + (int64_t)u * THREADS);
}

template <typename T, int U>
__device__ __forceinline__ void scale_all(uint4 (&v)[U], float s) {
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = scale_vec<T>(v[u], s);
}

// Forward chunk load; SCALED applies the logit scale to the loaded vectors.
template <typename T, bool SCALED, int U, int THREADS>
__device__ __forceinline__ void load_fwd(uint4 (&v)[U], const uint4* vp, int64_t j, float s) {
    load_vectors<U, THREADS>(v, vp, j);
    if constexpr (SCALED) {
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = scale_vec<T>(v[u], s);
    }
}

// Predicated chunk load: vectors at or beyond j1 read as padding (the dtype's lowest
// finite value, which adds exp(-huge) = 0 and is counted like any sub-maximum logit).
// SCALED scales the loaded vectors, never the padding.
template <typename T, int U, int THREADS, bool SCALED = false>
__device__ __forceinline__ void load_vectors_masked(uint4 (&v)[U], const uint4* vp, int64_t j,
                                                    int64_t j1, float s = 1.f) {
    const uint32_t pw = DT<T>::kPadWord;
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t jj = j + (int64_t)u * THREADS;
        if (jj < j1) {
            v[u] = ldg_stream(vp + jj);
            if constexpr (SCALED) v[u] = scale_vec<T>(v[u], s);
        } else {
            v[u] = make_uint4(pw, pw, pw, pw);
        }
    }
}

// The remainder of a segment (fewer than U vectors left for this thread): all its loads
// are issued at once, then reduced two vectors at a time, so it costs one memory round
// trip and no arithmetic on padding beyond one vector.
template <typename T, bool SCALED, int THREADS, int U>
__device__ __forceinline__ void fwd_remainder(const uint4* vp, int64_t j, int64_t j1,
                                              FwdState& st, bool clamp, float s) {
    uint4 v[U];
    load_vectors_masked<T, U, THREADS, SCALED>(v, vp, j, j1, s);
#pragma unroll
    for (int u = 0; u < U; u += 2) {
        if (j + (int64_t)u * THREADS < j1) {
            uint4 w[2] = {v[u], v[u + 1]};
            fwd_chunk<T, 2>(w, st, clamp);
        }
    }
}

// Stream vectors [j0, j1) of one row (vector path: row start 16-byte aligned and the
// row an exact number of vectors).  `tid` / THREADS: this thread's lane in the group
// that shares the segment.  With K1_FWD_PREFETCH the next chunk's loads are in flight
// while the current chunk is reduced (two register buffers used alternately): warps that
// start in lock-step (every warp of the grid issues its first loads together) would
// otherwise alternate between waiting for memory and computing instead of overlapping.
template <typename T, bool SCALED, int THREADS, int U, bool PF = (K1_FWD_PREFETCH != 0)>
__device__ __forceinline__ void fwd_stream_vec(const T* rowp, int64_t j0, int64_t j1,
                                               FwdState& st, int tid, bool clamp, float s) {
    const uint4* vp = reinterpret_cast<const uint4*>(rowp);
    constexpr int64_t kSpan = (int64_t)(U - 1) * THREADS;
    constexpr int64_t kStep = (int64_t)U * THREADS;
    int64_t j = j0 + tid;
    if constexpr (PF) {
        // raw loads go out a chunk ahead; the scale is applied when a chunk is consumed
        // (applying it at load time would wait for the loads right away)
        if (j + kSpan < j1) {
            uint4 a[U], b[U];
            load_vectors<U, THREADS>(a, vp, j);
            while (true) {
                bool more = j + kStep + kSpan < j1;
                if (more) load_vectors<U, THREADS>(b, vp, j + kStep);
                if constexpr (SCALED) scale_all<T, U>(a, s);
                fwd_chunk<T, U>(a, st, clamp);
                j += kStep;
                if (!more) break;
                more = j + kStep + kSpan < j1;
                if (more) load_vectors<U, THREADS>(a, vp, j + kStep);
                if constexpr (SCALED) scale_all<T, U>(b, s);
                fwd_chunk<T, U>(b, st, clamp);
                j += kStep;
                if (!more) break;
            }
        }
    } else {
        for (; j + kSpan < j1; j += kStep) {
            uint4 v[U];
            load_fwd<T, SCALED, U, THREADS>(v, vp, j, s);
            fwd_chunk<T, U>(v, st, clamp);
        }
    }
    if (j < j1) fwd_remainder<T, SCALED, THREADS, U>(vp, j, j1, st, clamp, s);
}

// Rows whose start is not 16-byte aligned (a vocabulary that is not a whole number of
// vectors, or such a row stride): a segment [j0, j1) is peeled into a head of single
// elements up to the first 16-byte boundary, an aligned interior of vectors and a tail of
// single elements.  Returns the interior [a0, a1) (a0 = a1 when there is none).
template <typename T>
__device__ __forceinline__ void peel(const T* rowp, int64_t j0, int64_t j1, int64_t& a0,
                                     int64_t& a1) {
    constexpr int EPV = DT<T>::kEPV;
    const uintptr_t a = reinterpret_cast<uintptr_t>(rowp + j0);
    const int64_t head = min((int64_t)(((16u - (unsigned)(a & 15u)) & 15u) / sizeof(T)), j1 - j0);
    a0 = j0 + head;
    a1 = a0 + (j1 - a0) / EPV * EPV;
}

// Stream elements [j0, j1) of one row at any alignment: the aligned interior through the
// vector path, the (at most 2 * (EPV - 1)) head and tail elements one per thread, each
// folded in as a pair with padding (the padding adds e = 0 like any masked element).
// Single elements are always clamped; `clamp` applies to the interior as on the vector path.
template <typename T, bool SCALED, int THREADS, int U>
__device__ __forceinline__ void fwd_stream_peeled(const T* rowp, int64_t j0, int64_t j1,
                                                  FwdState& st, int tid, bool clamp, float s) {
    using D = DT<T>;
    int64_t a0, a1;
    peel(rowp, j0, j1, a0, a1);
    if (a1 > a0)
        fwd_stream_vec<T, SCALED, THREADS, U>(rowp + a0, 0, (a1 - a0) / D::kEPV, st, tid, clamp,
                                              s);
    const int64_t nh = a0 - j0, ne = nh + (j1 - a1);
    if (tid < ne) {
        const int64_t e = tid < nh ? j0 + tid : a1 + (tid - nh);
        const float x = D::load1(rowp + e);
        const float xv = D::clamp1(SCALED ? scale1<T>(x, s) : x);
        st.rescale(xv);
        st.accum(make_float2(xv, D::kLowest), splat(-st.m));
        st.np += 1.f;
    }
}

template <typename T, bool SHARD>
__device__ __forceinline__ void fwd_emit_row(const FwdParams& p, int64_t r, const T* rowp,
                                             RowPartial part) {
    const int64_t tg = p.targets[r];
    if constexpr (SHARD) {
        const int64_t tl = tg - p.col_offset;
        const bool has = (tg >= 0) && (tl >= 0) && (tl < p.vocab);
        k1_partial out;
        out.z = part.z;
        out.t = part.t;
        out.m = part.m;
        out.x_t = has ? target_logit<T>(rowp + tl, p.scale) : 0.f;
        out.has_target = has ? 1 : 0;
        out.reserved = 0;
        p.partials[r] = out;
    } else {
        double xt = (tg >= 0 && tg < p.vocab) ? (double)target_logit<T>(rowp + tg, p.scale) : 0.0;
        finalize_row(part, xt, p.logprob + r, p.entropy + r, p.lse + r);
    }
}

// Rows a block finishes are not written immediately: their merged state is parked in
// shared memory and kRowCap rows are finalised at once, one row per thread (fp64 log and
// divide, the target-logit load).  Doing it per row in one thread would stall that warp,
// and with it the next block-wide barrier, once per row.
constexpr int kRowCap = 32;

template <int THREADS>
struct FwdSmem {
    static constexpr int NW = THREADS / 32;
    float wmax[2][NW];   // per-warp maxima, double-buffered by segment parity
    int wbad[2][NW];     // per-warp "saw -inf on the fast path"
    double wz[2][NW];
    double wt[2][NW];
    RowPartial done_part[kRowCap];
    int64_t done_row[kRowCap];
    unsigned split_prev[2];  // ticket values of the owner's first / last split row
    unsigned next_chunk[2];  // next dynamic chunk, double-buffered by grab parity
};

// Merge the threads' states of one segment into `out` (relative to the segment maximum).
// Returns false -- uniformly, after an extra barrier -- when some thread flagged `bad`; the
// caller then re-streams the segment clamped and merges again.  Two barriers otherwise:
// the scratch is double-buffered by segment parity, so no trailing barrier is needed.
template <int THREADS, int BAR>
__device__ __forceinline__ bool seg_merge(float m, double z, double t, bool empty, bool bad,
                                          FwdSmem<THREADS>& sm, int buf, RowPartial& out) {
    constexpr int NW = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float wm = warp_max_nan(empty ? -INFINITY : m);
    const bool wb = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        sm.wmax[buf][warp] = wm;
        sm.wbad[buf][warp] = wb ? 1 : 0;
    }
    group_sync<THREADS, BAR>();
    int any_bad = 0;
    float M = sm.wmax[buf][0];
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        any_bad |= sm.wbad[buf][i];
        M = fmax_nan(M, sm.wmax[buf][i]);
    }
    if (any_bad) {
        group_sync<THREADS, BAR>();  // everyone has read the flags before the retry
        return false;
    }
    double zc = 0.0, tc = 0.0;
    if (!empty) {
        const float dm = m - M;
        const float sc = (dm == 0.f) ? 1.f : ex2(dm * kLog2e);
        zc = (double)sc * z;
        tc = (double)sc * (t + (double)dm * z);
    }
    zc = warp_sum(zc);
    tc = warp_sum(tc);
    if (lane == 0) {
        sm.wz[buf][warp] = zc;
        sm.wt[buf][warp] = tc;
    }
    group_sync<THREADS, BAR>();
    out.z = 0.0;
    out.t = 0.0;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        out.z += sm.wz[buf][i];
        out.t += sm.wt[buf][i];
    }
    out.m = M;
    if (M == -INFINITY) out.z = out.t = 0.0;
    out.pad = 0.f;
    return true;
}

// Finalise the parked rows, one per thread.
template <typename T, int THREADS, int BAR, bool SHARD>
__device__ __forceinline__ void fwd_flush_rows(const FwdParams& p, FwdSmem<THREADS>& sm, int count) {
    group_sync<THREADS, BAR>();
    const int tid = threadIdx.x;
    if (tid < count) {
        const int64_t r = sm.done_row[tid];
        fwd_emit_row<T, SHARD>(p, r, reinterpret_cast<const T*>(p.logits) + p.lay.offset(r),
                               sm.done_part[tid]);
    }
    group_sync<THREADS, BAR>();
}

// Split row r (its units span owners bf..bl): merge every owner's published part and
// write the row.  Called by the block whose owner drew the last ticket; one
// warp does the work with shuffles (no block barrier), lane 0 issues the target-logit
// load first so that its latency overlaps the loads of the pieces.
template <typename T, bool SHARD>
__device__ __forceinline__ void fwd_merge_split_row(const FwdParams& p, int64_t r) {
    const int lane = threadIdx.x & 31;
    const Partition P = p.part();
    const int64_t bf = P.owner_of(r * p.vpr);
    const int64_t bl = P.owner_of((r + 1) * p.vpr - 1);
    const T* rowp = reinterpret_cast<const T*>(p.logits) + p.lay.offset(r);
    float xt = 0.f;
    bool has = false;
    if (lane == 0) {
        const int64_t tg = p.targets[r];
        const int64_t tl = SHARD ? tg - p.col_offset : tg;
        has = (tg >= 0) && (tl >= 0) && (tl < p.vocab);
        if (has) xt = target_logit<T>(rowp + tl, p.scale);
    }
    __threadfence();
    RowPartial acc;
    acc.z = 0.0;
    acc.t = 0.0;
    acc.m = -INFINITY;
    acc.pad = 0.f;
    for (int64_t c = bf + lane; c <= bl; c += 32) {
        const int64_t fr = P.start(c) / p.vpr;
        const RowPartial* q = p.ws_part + 2 * c + (r == fr ? 0 : 1);
        RowPartial qq;
        qq.z = __ldcg(&q->z);
        qq.t = __ldcg(&q->t);
        qq.m = __ldcg(&q->m);
        qq.pad = 0.f;
        acc = merge_partials(acc, qq);
    }
    // warp merge: common maximum first, one scale factor per lane, then plain fp64 sums
    const float M = warp_max_nan(acc.m);
    double zc = 0.0, tc = 0.0;
    if (acc.m != -INFINITY) {
        const float dm = acc.m - M;  // <= 0, NaN if either is NaN
        const float sc = (dm == 0.f) ? 1.f : ex2(dm * kLog2e);
        zc = (double)sc * acc.z;
        tc = (double)sc * (acc.t + (double)dm * acc.z);
    }
    acc.z = warp_sum(zc);
    acc.t = warp_sum(tc);
    acc.m = M;
    if (M == -INFINITY) acc.z = acc.t = 0.0;
    if (lane == 0) {
        if constexpr (SHARD) {
            k1_partial out;
            out.z = acc.z;
            out.t = acc.t;
            out.m = acc.m;
            out.x_t = has ? xt : 0.f;
            out.has_target = has ? 1 : 0;
            out.reserved = 0;
            p.partials[r] = out;
        } else {
            finalize_row(acc, has ? (double)xt : 0.0, p.logprob + r, p.entropy + r, p.lse + r);
        }
        p.ws_ticket[bf] = 0u;  // leave the workspace zeroed for the next call
    }
}

// Merge the split rows (first / last row of an owner, -1 = none) for which the owner drew
// the last ticket: the first by warp 0, the last by warp 1.  split_prev must be in shared
// memory and visible to those warps (a barrier after thread 0 wrote it).
template <typename T, int THREADS, bool SHARD>
__device__ __forceinline__ void fwd_merge_owner_rows(const FwdParams& p, const Partition& P,
                                                     const int64_t (&split_row)[2],
                                                     const FwdSmem<THREADS>& sm) {
    const int slot = threadIdx.x >> 5;
    if (slot < 2) {
        const int64_t sr = slot == 0 ? split_row[0] : split_row[1];
        if (sr >= 0) {
            const int64_t bf = P.owner_of(sr * p.vpr);
            const int64_t bl = P.owner_of((sr + 1) * p.vpr - 1);
            const unsigned prev = slot == 0 ? sm.split_prev[0] : sm.split_prev[1];
            if (prev == (unsigned)(bl - bf)) fwd_merge_split_row<T, SHARD>(p, sr);
        }
    }
}

// One owner's units (a block's static piece or a dynamic chunk): stream its row segments,
// park whole rows for the batched flush and publish partials of rows shared with other
// owners.  MERGE_NOW merges those for which this owner drew the last ticket before
// returning (two barriers, only when the owner has such rows); otherwise the split rows
// and their tickets (thread 0) are left in split_row / split_prev for the caller.
template <typename T, int THREADS, int U, bool VEC, bool SHARD, bool SCALED, bool MERGE_NOW>
__device__ __forceinline__ void fwd_owner(const FwdParams& p, const Partition& P, int64_t owner,
                                          FwdSmem<THREADS>& sm, int& count, int& buf,
                                          int64_t (&split_row)[2], unsigned (&split_prev)[2]) {
    constexpr int BAR = 0;
    const int tid = threadIdx.x;
    int64_t start = P.start(owner);
    const int64_t end = P.start(owner + 1);
    int64_t r = start / p.vpr;
    int64_t j0 = start - r * p.vpr;
    const int64_t first_row = r;
    split_row[0] = split_row[1] = -1;
    split_prev[0] = split_prev[1] = 0u;

    while (start < end) {
        const int64_t j1 = min(p.vpr, j0 + (end - start));
        const T* rowp = reinterpret_cast<const T*>(p.logits) + p.lay.offset(r);
        FwdState st;
        RowPartial part;
        if constexpr (VEC) {
            // second pass only when the segment holds -inf logits: stream it again, clamped
            for (int pass = 0; pass < 2; ++pass) {
                st.init();
                fwd_stream_vec<T, SCALED, THREADS, U>(rowp, j0, j1, st, tid, pass == 1, p.scale);
                if (seg_merge<THREADS, BAR>(st.m, st.z64(), st.t64(), st.m <= DT<T>::kLowest,
                                            pass == 0 && st.saw_neg_inf(), sm, buf, part))
                    break;
            }
        } else {
            for (int pass = 0; pass < 2; ++pass) {
                st.init();
                // 4 vectors a thread per chunk: this kernel is at its register budget
                fwd_stream_peeled<T, SCALED, THREADS, 4>(rowp, j0, j1, st, tid, pass == 1,
                                                         p.scale);
                if (seg_merge<THREADS, BAR>(st.m, st.z64(), st.t64(), st.m <= DT<T>::kLowest,
                                            pass == 0 && st.saw_neg_inf(), sm, buf, part))
                    break;
            }
        }
        buf ^= 1;
        if (j0 == 0 && j1 == p.vpr) {
            if (tid == 0) {
                sm.done_row[count] = r;
                sm.done_part[count] = part;
            }
            if (++count == kRowCap) {
                fwd_flush_rows<T, THREADS, BAR, SHARD>(p, sm, count);
                count = 0;
            }
        } else {
            // Row shared with other owners: publish this owner's part and draw a ticket;
            // the owner that draws the last one merges the row.
            const int slot = (r == first_row) ? 0 : 1;
            split_row[slot] = r;
            if (tid == 0) {
                p.ws_part[2 * owner + slot] = part;
                __threadfence();
                split_prev[slot] = atomicAdd(p.ws_ticket + P.owner_of(r * p.vpr), 1u);
            }
        }
        start += j1 - j0;
        ++r;
        j0 = 0;
    }
    if constexpr (MERGE_NOW) {
        if (split_row[0] < 0 && split_row[1] < 0) return;  // block-uniform
        if (tid == 0) {
            sm.split_prev[0] = split_prev[0];
            sm.split_prev[1] = split_prev[1];
        }
        group_sync<THREADS, BAR>();
        fwd_merge_owner_rows<T, THREADS, SHARD>(p, P, split_row, sm);
        group_sync<THREADS, BAR>();  // split_prev is rewritten by the next owner
    }
}

template <typename T, int THREADS, int U, bool VEC, bool SHARD, bool SCALED = false>
__global__ void __launch_bounds__(THREADS, K1_FWD_MINB) k1_fwd_kernel(FwdParams p) {
    constexpr int BAR = 0;
    __shared__ FwdSmem<THREADS> sm;
    pdl_wait();
    pdl_trigger();
    const Partition P = p.part();
    const int tid = threadIdx.x;
    int count = 0, buf = 0;
    // the block's static piece; its split rows are merged at the very end, after the
    // flush barrier (no extra barrier)
    int64_t srow[2];
    unsigned sprev[2];
    if (P.D == 0) {
        fwd_owner<T, THREADS, U, VEC, SHARD, SCALED, false>(p, P, blockIdx.x, sm, count, buf,
                                                            srow, sprev);
    } else {
        // the static piece, then dynamic chunks; the next chunk's index is requested when
        // an owner starts, so the atomic's latency overlaps that owner's streaming
        unsigned next = 0u;
        if (tid == 0) next = atomicAdd(p.ws_dyn, 1u);
        fwd_owner<T, THREADS, U, VEC, SHARD, SCALED, false>(p, P, blockIdx.x, sm, count, buf,
                                                            srow, sprev);
        int64_t owner = -1;
        int nb = 0;
        while (true) {
            if (owner >= 0) {
                int64_t drow[2];
                unsigned dprev[2];
                fwd_owner<T, THREADS, U, VEC, SHARD, SCALED, true>(p, P, owner, sm, count, buf,
                                                                   drow, dprev);
            }
            if (tid == 0) sm.next_chunk[nb] = next;
            group_sync<THREADS, BAR>();
            const unsigned o = sm.next_chunk[nb];
            nb ^= 1;
            if (o >= (unsigned)P.D) break;
            if (tid == 0) next = atomicAdd(p.ws_dyn, 1u);
            owner = P.G + o;
        }
        // the last block out leaves the counters zeroed for the next call
        if (tid == 0 && atomicAdd(p.ws_dyn + 1, 1u) == gridDim.x - 1) {
            p.ws_dyn[0] = 0u;
            p.ws_dyn[1] = 0u;
        }
    }
    if (tid == 0) {
        sm.split_prev[0] = sprev[0];
        sm.split_prev[1] = sprev[1];
    }
    fwd_flush_rows<T, THREADS, BAR, SHARD>(p, sm, count);  // its barrier publishes split_prev
    fwd_merge_owner_rows<T, THREADS, SHARD>(p, P, srow, sm);
}

// ---------------------------------------------------------------------------------
// Forward, row groups (many rows of moderate width): each group of GT threads (one, two
// or four warps) takes whole rows from a global queue (an atomic counter) and reduces
// each row on its own -- warp shuffles, plus a named barrier per group when GT > 32 --
// so rows are never split between owners and no block-wide barrier is taken.  Rows are
// handed out in order and a row is computed the same way by any group, so results do
// not depend on which group took it.  The next row's index is requested, and the row's
// target logit loaded, while the current row streams.
// ---------------------------------------------------------------------------------
template <int GT>
struct RowsSmem {
    static constexpr int NW = GT / 32;
    float wmax[2][NW];
    int wbad[2][NW];
    double wz[2][NW];
    double wt[2][NW];
};

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Merge the group's per-thread states of one row (relative to the row maximum).  Returns
// false -- uniformly -- when some thread flagged `bad`; the caller re-streams clamped.
template <int GT>
__device__ __forceinline__ bool rows_merge(float m, double z, double t, bool empty, bool bad,
                                           RowsSmem<GT>& sm, int bar_id, int wig, int buf,
                                           RowPartial& out) {
    constexpr int NW = GT / 32;
    const int lane = threadIdx.x & 31;
    float M = warp_max_nan(empty ? -INFINITY : m);
    bool any_bad = __any_sync(0xffffffffu, bad);
    if constexpr (NW > 1) {
        if (lane == 0) {
            sm.wmax[buf][wig] = M;
            sm.wbad[buf][wig] = any_bad ? 1 : 0;
        }
        named_sync(bar_id, GT);
        M = sm.wmax[buf][0];
        int b = sm.wbad[buf][0];
#pragma unroll
        for (int i = 1; i < NW; ++i) {
            M = fmax_nan(M, sm.wmax[buf][i]);
            b |= sm.wbad[buf][i];
        }
        any_bad = b != 0;
    }
    if (any_bad) {
        if constexpr (NW > 1) named_sync(bar_id, GT);  // flags read before the retry
        return false;
    }
    double zc = 0.0, tc = 0.0;
    if (!empty) {
        const float dm = m - M;
        const float sc = (dm == 0.f) ? 1.f : ex2(dm * kLog2e);
        zc = (double)sc * z;
        tc = (double)sc * (t + (double)dm * z);
    }
    zc = warp_sum(zc);
    tc = warp_sum(tc);
    if constexpr (NW > 1) {
        if (lane == 0) {
            sm.wz[buf][wig] = zc;
            sm.wt[buf][wig] = tc;
        }
        named_sync(bar_id, GT);
        zc = 0.0;
        tc = 0.0;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            zc += sm.wz[buf][i];
            tc += sm.wt[buf][i];
        }
    }
    out.z = zc;
    out.t = tc;
    out.m = M;
    if (M == -INFINITY) out.z = out.t = 0.0;
    out.pad = 0.f;
    return true;
}

template <typename T, int GT, int U, bool VEC, bool SHARD, bool SCALED>
__global__ void __launch_bounds__(256, K1_FWD_MINB) k1_fwd_rows_kernel(FwdParams p) {
    constexpr int NG = 256 / GT;
    __shared__ RowsSmem<GT> gsm[NG];
    __shared__ int64_t gnext[NG][2];
    pdl_wait();
    pdl_trigger();
    const int g = threadIdx.x / GT, gtid = threadIdx.x % GT, wig = gtid >> 5;
    const int bar_id = 1 + g;
    RowsSmem<GT>& sm = gsm[g];
    const unsigned n_groups = gridDim.x * NG;
    unsigned next = 0u;
    if (gtid == 0) next = atomicAdd(p.ws_dyn, 1u);
    int buf = 0, nb = 0;
    while (true) {
        // the group's next row (thread 0 of the group drew it)
        int64_t r;
        if constexpr (GT == 32) {
            r = (int64_t)__shfl_sync(0xffffffffu, next, 0);
        } else {
            if (gtid == 0) gnext[g][nb] = (int64_t)next;
            named_sync(bar_id, GT);
            r = gnext[g][nb];
            nb ^= 1;
        }
        if (r >= p.n_rows) break;
        const T* rowp = reinterpret_cast<const T*>(p.logits) + p.lay.offset(r);
        int64_t tg = -1;
        if (gtid == 0) {
            next = atomicAdd(p.ws_dyn, 1u);  // the row after this one
            tg = p.targets[r];               // consumed after the row has streamed
        }
        float xt = 0.f;
        bool has = false;
        FwdState st;
        RowPartial part;
        for (int pass = 0; pass < 2; ++pass) {
            st.init();
            if constexpr (VEC)
                fwd_stream_vec<T, SCALED, GT, U>(rowp, 0, p.vpr, st, gtid, pass == 1, p.scale);
            else
                fwd_stream_peeled<T, SCALED, GT, U>(rowp, 0, p.vpr, st, gtid, pass == 1, p.scale);
            if (gtid == 0) {  // the target logit's load overlaps the merge
                const int64_t tl = SHARD ? tg - p.col_offset : tg;
                has = (tg >= 0) && (tl >= 0) && (tl < p.vocab);
                xt = has ? target_logit<T>(rowp + tl, p.scale) : 0.f;
            }
            const bool ok = rows_merge<GT>(st.m, st.z64(), st.t64(), st.m <= DT<T>::kLowest,
                                           pass == 0 && st.saw_neg_inf(), sm, bar_id, wig, buf,
                                           part);
            buf ^= 1;
            if (ok) break;
        }
        if (gtid == 0) {
            if constexpr (SHARD) {
                k1_partial o;
                o.z = part.z;
                o.t = part.t;
                o.m = part.m;
                o.x_t = has ? xt : 0.f;
                o.has_target = has ? 1 : 0;
                o.reserved = 0;
                p.partials[r] = o;
            } else {
                finalize_row(part, has ? (double)xt : 0.0, p.logprob + r, p.entropy + r,
                             p.lse + r);
            }
        }
    }
    // the last group out leaves the counters zeroed for the next call
    if (gtid == 0 && atomicAdd(p.ws_dyn + 1, 1u) == n_groups - 1) {
        p.ws_dyn[0] = 0u;
        p.ws_dyn[1] = 0u;
    }
}

// ---------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------
struct BwdRow {
    float lse, ent, gl, ge, gs, c0;
    int64_t tl;  // target column inside this row, or -1
};

// Gradient of the target column in fp64: g_logp (1 - p) + p (g_lse - g_ent (log p + H)),
// with 1 - p = -expm1(log p), so a confident target (p -> 1) keeps its relative accuracy.
__device__ __forceinline__ float bwd_target_value(float x, const BwdRow& q) {
    double dt = (double)x - (double)q.lse;
    double pt = exp(dt);
    if (pt == 0.0) return q.gl;
    double om = -expm1(dt);
    return (float)((double)q.gl * om + pt * ((double)q.gs - (double)q.ge * (dt + (double)q.ent)));
}

// Gradient w.r.t. the stored target logit of row xr: the value above at the scaled logit,
// rounded to the logits' type, times the scale (both identities at scale 1).
template <typename T>
__device__ __forceinline__ float bwd_target_out(const T* xr, const BwdRow& q, float s) {
    return scale1<T>(DT<T>::round1(bwd_target_value(target_logit<T>(xr + q.tl, s), q)), s);
}

template <typename T, bool SCALED = false>
__device__ __forceinline__ uint4 bwd_vector(uint4 v, const BwdRow& q, float s = 1.f) {
    using D = DT<T>;
    if constexpr (SCALED) v = scale_vec<T>(v, s);
    const float2 nl = splat(-q.lse), c02 = splat(q.c0), nge = splat(-q.ge);
    uint4 o;
    if constexpr (sizeof(T) == 2) {
        uint32_t in[4] = {v.x, v.y, v.z, v.w};
        uint32_t out[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 x = D::to_f2(D::clamp2(in[i]));
            float2 d = add2(x, nl);
            float2 tt = mul2(d, splat(kLog2e));
            float2 pp = make_float2(ex2(tt.x), ex2(tt.y));
            float2 g = fma2(nge, mul2(pp, d), mul2(pp, c02));
            out[i] = D::from_f2(g);
        }
        o = make_uint4(out[0], out[1], out[2], out[3]);
    } else {
        float in[4] = {__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z),
                       __uint_as_float(v.w)};
        float out[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            float2 x = make_float2(D::clamp1(in[2 * i]), D::clamp1(in[2 * i + 1]));
            float2 d = add2(x, nl);
            float2 tt = mul2(d, splat(kLog2e));
            float2 pp = make_float2(ex2(tt.x), ex2(tt.y));
            float2 g = fma2(nge, mul2(pp, d), mul2(pp, c02));
            out[2 * i] = g.x;
            out[2 * i + 1] = g.y;
        }
        o = make_uint4(__float_as_uint(out[0]), __float_as_uint(out[1]), __float_as_uint(out[2]),
                       __float_as_uint(out[3]));
    }
    if constexpr (SCALED) o = scale_vec<T>(o, s);  // o already holds dtype(dL/dy)
    return o;
}

// Replace element k of a packed vector by `val` (k known only at run time; unrolled
// selects keep the vector in registers).
template <typename T>
__device__ __forceinline__ uint4 vec_set(uint4 o, int k, float val) {
    using D = DT<T>;
    uint32_t w[4] = {o.x, o.y, o.z, o.w};
    if constexpr (sizeof(T) == 2) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if ((k >> 1) == i) {
                float2 f = D::to_f2(w[i]);
                if (k & 1) f.y = val; else f.x = val;
                w[i] = D::from_f2(f);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (k == i) w[i] = __float_as_uint(val);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Gradient of vectors [j0, j1) of a row through a 16-byte aligned vector base xv / dv.
// tl_rel is the target column relative to the base's first element (outside [0, vectors
// x EPV) when the target is elsewhere); xr is the row's first element.
template <typename T, bool SCALED, int THREADS, int U>
__device__ __forceinline__ void bwd_stream_vec(const uint4* xv, uint4* dv, int64_t j0, int64_t j1,
                                               const BwdRow& q, int64_t tl_rel, const T* xr,
                                               float s) {
    constexpr int EPV = DT<T>::kEPV;
    constexpr int64_t kSpan = (int64_t)(U - 1) * THREADS;
    constexpr int64_t kStep = (int64_t)U * THREADS;
    int64_t j = j0 + threadIdx.x;
    for (; j + kSpan < j1; j += kStep) {
        uint4 v[U];
        load_vectors<U, THREADS>(v, xv, j);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t jj = j + (int64_t)u * THREADS;
            uint4 o = bwd_vector<T, SCALED>(v[u], q, s);
            const uint64_t k = (uint64_t)(tl_rel - jj * EPV);
            if (k < (uint64_t)EPV) o = vec_set<T>(o, (int)k, bwd_target_out<T>(xr, q, s));
            stg_stream(dv + jj, o);
        }
    }
    if (j < j1) {  // remainder: one predicated chunk
        uint4 v[U];
        load_vectors_masked<T, U, THREADS>(v, xv, j, j1);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t jj = j + (int64_t)u * THREADS;
            if (jj < j1) {
                uint4 o = bwd_vector<T, SCALED>(v[u], q, s);
                const uint64_t k = (uint64_t)(tl_rel - jj * EPV);
                if (k < (uint64_t)EPV) o = vec_set<T>(o, (int)k, bwd_target_out<T>(xr, q, s));
                stg_stream(dv + jj, o);
            }
        }
    }
}

// Gradient of the single element j of a row: the packed path's operations one lane at a
// time, so both paths produce identical bits.
template <typename T, bool SCALED>
__device__ __forceinline__ void bwd_element(const T* xr, T* dr, int64_t j, const BwdRow& q,
                                            float s) {
    using D = DT<T>;
    float g;
    if (j == q.tl) {
        g = bwd_target_out<T>(xr, q, s);
    } else {
        const float xraw = D::load1(xr + j);
        const float x = D::clamp1(SCALED ? scale1<T>(xraw, s) : xraw);
        const float d = __fadd_rn(x, -q.lse);
        const float pp = ex2(__fmul_rn(d, kLog2e));
        g = __fmaf_rn(-q.ge, __fmul_rn(pp, d), __fmul_rn(pp, q.c0));
        if constexpr (SCALED) g = scale1<T>(D::round1(g), s);
    }
    D::store1(dr + j, g);
}

template <typename T, int THREADS, int U, bool VEC, bool SCALED = false>
__global__ void __launch_bounds__(THREADS, K1_BWD_MINB) k1_bwd_kernel(BwdParams p) {
    using D = DT<T>;
    constexpr int EPV = D::kEPV;
    pdl_wait();
    pdl_trigger();
    const int64_t G = gridDim.x, b = blockIdx.x;
    int64_t start = b * p.total / G;
    const int64_t end = (b + 1) * p.total / G;
    int64_t r = start / p.vpr;
    int64_t j0 = start - r * p.vpr;

    while (start < end) {
        const int64_t j1 = min(p.vpr, j0 + (end - start));
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
        if constexpr (VEC) {
            bwd_stream_vec<T, SCALED, THREADS, U>(reinterpret_cast<const uint4*>(xr),
                                                  reinterpret_cast<uint4*>(dr), j0, j1, q, q.tl,
                                                  xr, p.scale);
        } else {
            // Rows that are not whole vectors: when the logits row and the gradient row
            // share their 16-byte misalignment, the aligned interior goes through the vector
            // path and only the head and tail elements one at a time; otherwise every
            // element one at a time.
            int64_t a0 = j1, a1 = j1;
            const uintptr_t ax = reinterpret_cast<uintptr_t>(xr + j0);
            const uintptr_t ad = reinterpret_cast<uintptr_t>(dr + j0);
            if (((ax ^ ad) & 15u) == 0) peel(xr, j0, j1, a0, a1);
            if (a1 > a0)
                bwd_stream_vec<T, SCALED, THREADS, K1_BWD_PEEL_UNROLL>(reinterpret_cast<const uint4*>(xr + a0),
                                                      reinterpret_cast<uint4*>(dr + a0), 0,
                                                      (a1 - a0) / EPV, q, q.tl - a0, xr, p.scale);
            const int64_t nh = a0 - j0, ne = nh + (j1 - a1);
            for (int64_t e = threadIdx.x; e < ne; e += THREADS)
                bwd_element<T, SCALED>(xr, dr, e < nh ? j0 + e : a1 + (e - nh), q, p.scale);
        }
        start += j1 - j0;
        ++r;
        j0 = 0;
    }
}

// ---------------------------------------------------------------------------------
// Naive forward: one thread per row, two passes, fp64.  Correctness anchor only.
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void k1_naive_kernel(const T* logits, int64_t n_rows, int64_t vocab, RowLayout lay,
                                const int64_t* targets, float* logprob, float* entropy,
                                float* lse) {
    pdl_wait();
    pdl_trigger();
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    const T* row = logits + lay.offset(r);
    double m = -INFINITY;
    bool nan = false;
    for (int64_t v = 0; v < vocab; ++v) {
        double x = (double)DT<T>::load1(row + v);
        if (isnan(x)) nan = true;
        else if (x > m) m = x;
    }
    RowPartial part;
    part.pad = 0.f;
    if (nan || m == INFINITY) {
        part.m = __int_as_float(0x7fc00000);
        part.z = part.t = 0.0;
    } else if (m == -INFINITY) {
        part.m = -INFINITY;
        part.z = part.t = 0.0;
    } else {
        double z = 0.0, t = 0.0;
        for (int64_t v = 0; v < vocab; ++v) {
            double x = (double)DT<T>::load1(row + v);
            if (x == -INFINITY) continue;
            double d = x - m;
            double e = exp(d);
            z += e;
            t += e * d;
        }
        part.m = (float)m;
        part.z = z;
        part.t = t;
    }
    const int64_t tg = targets[r];
    double xt = (tg >= 0 && tg < vocab) ? (double)DT<T>::load1(row + tg) : 0.0;
    finalize_row(part, xt, logprob + r, entropy + r, lse + r);
}

// ---------------------------------------------------------------------------------
// Vocab-parallel combine: one thread per row over the gathered shard partials.
// ---------------------------------------------------------------------------------
__global__ void k1_vocab_combine_kernel(const k1_partial* g, int n_shards, int64_t n_rows,
                                        float* logprob, float* entropy, float* lse) {
    pdl_wait();
    pdl_trigger();
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    RowPartial acc;
    acc.z = 0.0;
    acc.t = 0.0;
    acc.m = -INFINITY;
    acc.pad = 0.f;
    double xt = 0.0;
    auto fold = [&](const k1_partial& q) {
        RowPartial pk;
        pk.z = q.z;
        pk.t = q.t;
        pk.m = q.m;
        pk.pad = 0.f;
        acc = merge_partials(acc, pk);
        if (q.has_target) xt = (double)q.x_t;
    };
    // up to kBatch shards' partials are loaded before the first merge (one memory round
    // trip instead of one per shard); the merge order is the shard order either way
    constexpr int kBatch = 8;
    for (int k0 = 0; k0 < n_shards; k0 += kBatch) {
        k1_partial q[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
            if (k0 + i < n_shards) q[i] = g[(int64_t)(k0 + i) * n_rows + r];
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
            if (k0 + i < n_shards) fold(q[i]);
    }
    finalize_row(acc, xt, logprob + r, entropy + r, lse + r);
}

}  // namespace k1
