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
#pragma once

#include "k1_common.cuh"
#include "../../include/k1_logprob.h"

namespace k1 {

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
    RowPartial* ws_part;   // 2 * gridDim.x slots
    unsigned* ws_ticket;   // gridDim.x counters, zero between calls
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
};

// Block that owns flattened unit u when `total` units are cut into G equal pieces
// (piece b = [floor(b * total / G), floor((b + 1) * total / G))).
__device__ __forceinline__ int64_t block_of(int64_t u, int64_t total, int64_t G) {
    return ((u + 1) * G + total - 1) / total - 1;
}

// ---------------------------------------------------------------------------------
// Forward: per-chunk work of one thread
// ---------------------------------------------------------------------------------
template <typename T, int U>
__device__ __forceinline__ void fwd_chunk(const uint4 (&v)[U], FwdState& st) {
    using D = DT<T>;
    if constexpr (sizeof(T) == 2) {
        uint32_t w[4 * U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            w[4 * u + 0] = D::clamp2(v[u].x);
            w[4 * u + 1] = D::clamp2(v[u].y);
            w[4 * u + 2] = D::clamp2(v[u].z);
            w[4 * u + 3] = D::clamp2(v[u].w);
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
        for (int i = 0; i < 4 * U; ++i) st.accum(D::to_f2(w[i]), nm);
    } else {
        float f[4 * U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            f[4 * u + 0] = D::clamp1(__uint_as_float(v[u].x));
            f[4 * u + 1] = D::clamp1(__uint_as_float(v[u].y));
            f[4 * u + 2] = D::clamp1(__uint_as_float(v[u].z));
            f[4 * u + 3] = D::clamp1(__uint_as_float(v[u].w));
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
    }
}

// Stream vectors [j0, j1) of one row (vector path: row start 16-byte aligned and the
// row an exact number of vectors).
template <typename T, int THREADS, int U>
__device__ __forceinline__ void fwd_stream_vec(const T* rowp, int64_t j0, int64_t j1,
                                               FwdState& st) {
    const uint4* vp = reinterpret_cast<const uint4*>(rowp);
    int64_t j = j0 + threadIdx.x;
    for (; j + (int64_t)(U - 1) * THREADS < j1; j += (int64_t)U * THREADS) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = ldg_stream(vp + j + (int64_t)u * THREADS);
        fwd_chunk<T, U>(v, st);
    }
    for (; j < j1; j += THREADS) {
        uint4 v[1];
        v[0] = ldg_stream(vp + j);
        fwd_chunk<T, 1>(v, st);
    }
}

// Stream elements [j0, j1) of one row (scalar path: any alignment).
template <typename T, int THREADS>
__device__ __forceinline__ void fwd_stream_scalar(const T* rowp, int64_t j0, int64_t j1,
                                                  FwdState& st) {
    using D = DT<T>;
    constexpr int U = 8;
    for (int64_t j = j0 + threadIdx.x; j < j1; j += (int64_t)U * THREADS) {
        float f[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int64_t jj = j + (int64_t)u * THREADS;
            f[u] = (jj < j1) ? D::clamp1(D::load1(rowp + jj)) : D::kLowest;
        }
        float mx = f[0];
#pragma unroll
        for (int u = 1; u < U; ++u) mx = fmax_nan(mx, f[u]);
        st.rescale(mx);
        const float2 nm = splat(-st.m);
#pragma unroll
        for (int i = 0; i < U / 2; ++i) st.accum(make_float2(f[2 * i], f[2 * i + 1]), nm);
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
        out.x_t = has ? DT<T>::load1(rowp + tl) : 0.f;
        out.has_target = has ? 1 : 0;
        out.reserved = 0;
        p.partials[r] = out;
    } else {
        double xt = (tg >= 0 && tg < p.vocab) ? (double)DT<T>::load1(rowp + tg) : 0.0;
        finalize_row(part, xt, p.logprob + r, p.entropy + r, p.lse + r);
    }
}

template <typename T, int THREADS, int U, bool VEC, bool SHARD>
__global__ void __launch_bounds__(THREADS) k1_fwd_kernel(FwdParams p) {
    __shared__ ReduceSmem<THREADS> sm;
    __shared__ int s_last;
    const int64_t G = gridDim.x, b = blockIdx.x;
    int64_t start = b * p.total / G;
    const int64_t end = (b + 1) * p.total / G;
    int64_t r = start / p.vpr;
    int64_t j0 = start - r * p.vpr;
    const int64_t first_row = r;

    while (start < end) {
        const int64_t j1 = min(p.vpr, j0 + (end - start));
        const T* rowp = reinterpret_cast<const T*>(p.logits) + p.lay.offset(r);
        FwdState st;
        st.init();
        if constexpr (VEC) {
            fwd_stream_vec<T, THREADS, U>(rowp, j0, j1, st);
        } else {
            fwd_stream_scalar<T, THREADS>(rowp, j0, j1, st);
        }
        const bool empty = st.m <= DT<T>::kLowest;  // false for NaN
        const double z = ((double)st.zb.x + (double)st.zb.y) + ((double)st.zs.x + (double)st.zs.y);
        const double t = (double)st.t.x + (double)st.t.y;
        RowPartial part = block_merge<THREADS>(st.m, z, t, empty, sm);

        if (j0 == 0 && j1 == p.vpr) {
            if (threadIdx.x == 0) fwd_emit_row<T, SHARD>(p, r, rowp, part);
        } else {
            // Row shared with neighbouring blocks: publish this block's piece, and the
            // last block to arrive merges all pieces.
            const int64_t bf = block_of(r * p.vpr, p.total, G);
            const int64_t bl = block_of((r + 1) * p.vpr - 1, p.total, G);
            if (threadIdx.x == 0) {
                RowPartial* slot = p.ws_part + 2 * b + (r == first_row ? 0 : 1);
                *slot = part;
                __threadfence();
                const unsigned prev = atomicAdd(p.ws_ticket + bf, 1u);
                s_last = (prev == (unsigned)(bl - bf)) ? 1 : 0;
            }
            __syncthreads();
            if (s_last) {
                __threadfence();
                RowPartial acc;
                acc.z = 0.0;
                acc.t = 0.0;
                acc.m = -INFINITY;
                acc.pad = 0.f;
                for (int64_t c = bf + threadIdx.x; c <= bl; c += THREADS) {
                    const int64_t fr = (c * p.total / G) / p.vpr;
                    const RowPartial* q = p.ws_part + 2 * c + (r == fr ? 0 : 1);
                    RowPartial qq;
                    qq.z = __ldcg(&q->z);
                    qq.t = __ldcg(&q->t);
                    qq.m = __ldcg(&q->m);
                    qq.pad = 0.f;
                    acc = merge_partials(acc, qq);
                }
                RowPartial tot = block_merge<THREADS>(acc.m, acc.z, acc.t,
                                                      acc.m == -INFINITY, sm);
                if (threadIdx.x == 0) {
                    fwd_emit_row<T, SHARD>(p, r, rowp, tot);
                    p.ws_ticket[bf] = 0u;  // leave the workspace zeroed for the next call
                }
            }
            __syncthreads();
        }
        start += j1 - j0;
        ++r;
        j0 = 0;
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

template <typename T>
__device__ __forceinline__ uint4 bwd_vector(uint4 v, const BwdRow& q) {
    using D = DT<T>;
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

template <typename T, int THREADS, int U, bool VEC>
__global__ void __launch_bounds__(THREADS) k1_bwd_kernel(BwdParams p) {
    using D = DT<T>;
    constexpr int EPV = VEC ? D::kEPV : 1;
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
            const uint4* xv = reinterpret_cast<const uint4*>(xr);
            uint4* dv = reinterpret_cast<uint4*>(dr);
            int64_t j = j0 + threadIdx.x;
            for (; j + (int64_t)(U - 1) * THREADS < j1; j += (int64_t)U * THREADS) {
                uint4 v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) v[u] = ldg_stream(xv + j + (int64_t)u * THREADS);
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t jj = j + (int64_t)u * THREADS;
                    uint4 o = bwd_vector<T>(v[u], q);
                    const uint64_t k = (uint64_t)(q.tl - jj * EPV);
                    if (k < (uint64_t)EPV)
                        o = vec_set<T>(o, (int)k, bwd_target_value(D::load1(xr + q.tl), q));
                    stg_stream(dv + jj, o);
                }
            }
            for (; j < j1; j += THREADS) {
                uint4 o = bwd_vector<T>(ldg_stream(xv + j), q);
                const uint64_t k = (uint64_t)(q.tl - j * EPV);
                if (k < (uint64_t)EPV)
                    o = vec_set<T>(o, (int)k, bwd_target_value(D::load1(xr + q.tl), q));
                stg_stream(dv + j, o);
            }
        } else {
            for (int64_t j = j0 + threadIdx.x; j < j1; j += THREADS) {
                const float xraw = D::load1(xr + j);
                float g;
                if (j == q.tl) {
                    g = bwd_target_value(xraw, q);
                } else {
                    const float x = D::clamp1(xraw);
                    const float d = x - q.lse;
                    const float pp = ex2(d * kLog2e);
                    g = pp * q.c0 - q.ge * (pp * d);
                }
                D::store1(dr + j, g);
            }
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
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    RowPartial acc;
    acc.z = 0.0;
    acc.t = 0.0;
    acc.m = -INFINITY;
    acc.pad = 0.f;
    double xt = 0.0;
    for (int k = 0; k < n_shards; ++k) {
        const k1_partial q = g[(int64_t)k * n_rows + r];
        RowPartial pk;
        pk.z = q.z;
        pk.t = q.t;
        pk.m = q.m;
        pk.pad = 0.f;
        acc = merge_partials(acc, pk);
        if (q.has_target) xt = (double)q.x_t;
    }
    finalize_row(acc, xt, logprob + r, entropy + r, lse + r);
}

}  // namespace k1
