// k1_common.cuh -- device building blocks shared by the K1 kernels (sm_100a).
//
// Streaming state.  The reference keeps one (m, Z, T) triple per thread and merges a
// one-element state into it for every logit, which costs two exponentials per element
// (csrc/fused_logprob.cu:141-154, 183-188).  Here a thread loads a chunk of logits,
// folds the chunk maximum with packed bf16x2 / f16x2 max instructions, rescales its
// state once per chunk, and then spends exactly one ex2 per element.  Arithmetic uses
// the Blackwell packed f32x2 add / mul / fma, two logits per instruction.
//
// Precision.  Z = sum exp(x - m) is kept as (count of logits equal to the running
// maximum) + (fp32 sum of the other terms).  A compare masks the maximum's own term (d =
// x - m is exactly 0 there) out of the fp32 sum, so for a near-one-hot row the tail keeps
// its full relative precision; a plain fp32 Z would be 1 + tail and round the tail (and
// with it the entropy) away.  Terms that only become "rest" when the maximum later moves
// are folded in scaled by exp(m_old - m_new), where a dominant new maximum makes them
// negligible and a close one makes the entropy large.  T = sum exp(x - m)(x - m) is a
// sum of non-positive terms, so it never cancels.  Thread and block states merge in fp64.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace k1 {

constexpr float kLog2e = 1.4426950408889634f;
// fp32 logits are clamped to this before use, so x - m stays finite for x = -inf.
constexpr float kClampF32 = -1.0e38f;

// ---------------------------------------------------------------------------------
// Scalar / packed primitives
// ---------------------------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 1.0f where d != 0 or d is NaN, else 0.0f.
__device__ __forceinline__ float not_zero(float d) {
    float y;
    asm("set.neu.f32.f32 %0, %1, 0f00000000;" : "=f"(y) : "f"(d));
    return y;
}

// Programmatic dependent launch.  Every K1 kernel is launched so that it may start
// before the previous kernel in the stream has finished; pdl_wait() then blocks until
// that kernel has completed and its writes are visible, and must come before the first
// global-memory access.  pdl_trigger() lets the next kernel in the stream be scheduled
// into the slots this grid frees as its blocks finish.  Both are no-ops for launches
// without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// NaN-propagating max (fmaxf drops NaN; the reference's outputs become NaN when a
// row holds one, and so do ours).
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float y;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(y) : "f"(a), "f"(b));
    return y;
}

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 splat(float v) { return make_float2(v, v); }
// a - b, exactly rounded (a single fma with -1).
__device__ __forceinline__ float2 diff2(float2 a, float2 b) { return fma2(b, splat(-1.f), a); }

// Streaming 16-byte load: read once, do not keep in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void stg_stream(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// ---------------------------------------------------------------------------------
// Element types.  A 16-byte vector holds kEPV elements; for the 16-bit types it is
// four 32-bit words of two elements each.
// ---------------------------------------------------------------------------------
template <typename T>
struct DT;

template <>
struct DT<__nv_bfloat16> {
    static constexpr int kEPV = 8;
    static constexpr uint32_t kLowest2 = 0xFF7FFF7Fu;  // lowest finite bf16, both halves
    static constexpr float kLowest = -3.38953138925153547590470800371487866880e38f;
    static constexpr uint32_t kPadWord = kLowest2;  // vector padding: contributes e = 0
    static constexpr uint32_t kNaNWord = 0x7FC07FC0u;  // quiet NaN, both halves
    __device__ static __forceinline__ uint32_t clamp2(uint32_t w) {
        uint32_t r;
        asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(w), "r"(kLowest2));
        return r;
    }
    __device__ static __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
        uint32_t r;
        asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
        return r;
    }
    __device__ static __forceinline__ float2 to_f2(uint32_t w) {
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
    __device__ static __forceinline__ uint32_t from_f2(float2 v) {
        uint32_t r;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(v.y), "f"(v.x));
        return r;
    }
    __device__ static __forceinline__ float load1(const __nv_bfloat16* p) {
        return __bfloat162float(*p);
    }
    __device__ static __forceinline__ void store1(__nv_bfloat16* p, float v) {
        *p = __float2bfloat16_rn(v);
    }
    __device__ static __forceinline__ float clamp1(float x) { return fmax_nan(x, kLowest); }
    __device__ static __forceinline__ float round1(float v) {
        return __bfloat162float(__float2bfloat16_rn(v));
    }
    // Both elements of w times s: fp32 products rounded to nearest-even bf16.
    __device__ static __forceinline__ uint32_t scale2(uint32_t w, float s) {
        return from_f2(mul2(to_f2(w), splat(s)));
    }
};

// d = x - m for the two bf16 logits of w, without a separate conversion: the sm_100
// mixed-precision add takes a bf16 operand and an fp32 operand.
__device__ __forceinline__ float2 bf16x2_minus(uint32_t w, float nm) {
    float d0, d1;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "add.rn.f32.bf16 %0, lo, %3;\n\tadd.rn.f32.bf16 %1, hi, %3;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "r"(w), "f"(nm));
    return make_float2(d0, d1);
}

// The same for two fp16 logits (f16 -> f32 is exact, the add rounds once: identical to
// converting first and subtracting in fp32).
__device__ __forceinline__ float2 f16x2_minus(uint32_t w, float nm) {
    float d0, d1;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "add.rn.f32.f16 %0, lo, %3;\n\tadd.rn.f32.f16 %1, hi, %3;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "r"(w), "f"(nm));
    return make_float2(d0, d1);
}

template <>
struct DT<__half> {
    static constexpr int kEPV = 8;
    static constexpr uint32_t kLowest2 = 0xFBFFFBFFu;  // -65504, both halves
    static constexpr float kLowest = -65504.0f;
    static constexpr uint32_t kPadWord = kLowest2;
    static constexpr uint32_t kNaNWord = 0x7E007E00u;  // quiet NaN, both halves
    __device__ static __forceinline__ uint32_t clamp2(uint32_t w) {
        uint32_t r;
        asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(w), "r"(kLowest2));
        return r;
    }
    __device__ static __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
        uint32_t r;
        asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
        return r;
    }
    __device__ static __forceinline__ float2 to_f2(uint32_t w) {
        __half2 h = *reinterpret_cast<__half2*>(&w);
        return __half22float2(h);
    }
    __device__ static __forceinline__ uint32_t from_f2(float2 v) {
        uint32_t r;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(v.y), "f"(v.x));
        return r;
    }
    __device__ static __forceinline__ float load1(const __half* p) { return __half2float(*p); }
    __device__ static __forceinline__ void store1(__half* p, float v) { *p = __float2half_rn(v); }
    __device__ static __forceinline__ float clamp1(float x) { return fmax_nan(x, kLowest); }
    __device__ static __forceinline__ float round1(float v) { return __half2float(__float2half_rn(v)); }
    // Both elements of w times s: fp32 products rounded to nearest-even fp16.
    __device__ static __forceinline__ uint32_t scale2(uint32_t w, float s) {
        return from_f2(mul2(to_f2(w), splat(s)));
    }
};

template <>
struct DT<float> {
    static constexpr int kEPV = 4;
    static constexpr float kLowest = kClampF32;
    static constexpr uint32_t kPadWord = 0xFE967699u;  // bits of -1.0e38f
    static constexpr uint32_t kNaNWord = 0x7FC00000u;  // quiet NaN
    __device__ static __forceinline__ float load1(const float* p) { return *p; }
    __device__ static __forceinline__ void store1(float* p, float v) { *p = v; }
    __device__ static __forceinline__ float clamp1(float x) { return fmax_nan(x, kClampF32); }
    __device__ static __forceinline__ float round1(float v) { return v; }
};

// ---------------------------------------------------------------------------------
// Forward streaming state of one thread (see the header comment).
// ---------------------------------------------------------------------------------
struct FwdState {
    float m;    // running maximum (clamped logits); <= kLowest of the type means "empty"
    float np;   // logits per lane since the running maximum last moved
    float2 zs;  // sum of exp(x - m) over logits below the running maximum
    float2 ms;  // number of logits below the running maximum since it last moved
    float2 t;   // sum of exp(x - m) * (x - m)

    __device__ __forceinline__ void init() {
        m = -3.402823466e38f;
        np = 0.f;
        zs = splat(0.f);
        ms = splat(0.f);
        t = splat(0.f);
    }

    // Logits equal to the running maximum, per lane.
    __device__ __forceinline__ float2 at_max() const { return make_float2(np - ms.x, np - ms.y); }

    // Move the reference point to max(m, mc).  Exact no-op when the maximum is unchanged.
    __device__ __forceinline__ void rescale(float mc) {
        const float mn = fmax_nan(m, mc);
        const float dl = m - mn;  // <= 0, or NaN
        const bool moved = !(dl == 0.f);
        const float s = moved ? ex2(dl * kLog2e) : 1.f;
        const float2 z = add2(zs, at_max());
        // t' = (t + dl z) s, evaluated as (dl s) z + t s: dl s stays within [-1/e, 0] for
        // any dl, whereas dl z overflows to -inf (and times s = 0 gives NaN) when the
        // first maximum was a clamped -inf (dl ~ -3.4e38) and several logits sat at it.
        t = fma2(splat(dl * s), z, mul2(t, splat(s)));
        if (moved) {
            zs = mul2(z, splat(s));
            ms = splat(0.f);
            np = 0.f;
        }
        m = mn;
    }

    // Accumulate two logits given as d = x - m; the caller adds the logits per lane to np
    // once per chunk.
    __device__ __forceinline__ void accum_d(float2 d) {
        const float2 tt = mul2(d, splat(kLog2e));
        const float2 e = make_float2(ex2(tt.x), ex2(tt.y));
        const float2 nz = make_float2(not_zero(d.x), not_zero(d.y));
        zs = fma2(e, nz, zs);
        ms = add2(ms, nz);
        t = fma2(e, d, t);
    }

    // Accumulate two logits; nm = (-m, -m).
    __device__ __forceinline__ void accum(float2 x, float2 nm) { accum_d(add2(x, nm)); }

    // Z of this thread in fp64 (count at the maximum + the rest).
    __device__ __forceinline__ double z64() const {
        const float2 c = at_max();
        return ((double)c.x + (double)c.y) + ((double)zs.x + (double)zs.y);
    }
    __device__ __forceinline__ double t64() const { return (double)t.x + (double)t.y; }

    // true when a -inf logit met the fast (unclamped) path: e = 0 times d = -inf made t
    // NaN while z stayed finite.  NaN logits poison z as well and are not flagged.
    __device__ __forceinline__ bool saw_neg_inf() const {
        return isnan(t.x + t.y) && !isnan(zs.x + zs.y) && !isnan(m);
    }
};

// Row (or row-segment) state after a block reduction, relative to its maximum m.
// m = -inf with z = t = 0 is the empty state (every logit -inf); NaN m poisons.
struct RowPartial {
    double z;
    double t;
    float m;
    float pad;
};

// ---------------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------------
__device__ __forceinline__ float warp_max_nan(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Barrier over the first THREADS threads of the block: the whole block (BAR = 0,
// __syncthreads) or a named hardware barrier shared by those threads only (BAR > 0,
// used when a producer warp does not take part).
template <int THREADS, int BAR>
__device__ __forceinline__ void group_sync() {
    if constexpr (BAR == 0) {
        __syncthreads();
    } else {
        asm volatile("bar.sync %0, %1;" ::"r"(BAR), "r"(THREADS) : "memory");
    }
}

template <int THREADS, int BAR>
__device__ __forceinline__ bool group_or(bool v) {
    if constexpr (BAR == 0) {
        return __syncthreads_or(v) != 0;
    } else {
        uint32_t r;
        asm volatile(
            "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
            "bar.red.or.pred po, %2, %3, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
            : "=r"(r)
            : "r"((uint32_t)v), "r"(BAR), "r"(THREADS)
            : "memory");
        return r != 0;
    }
}

// Shared scratch for one block reduction.
template <int THREADS>
struct ReduceSmem {
    float wmax[THREADS / 32];
    double wz[THREADS / 32];
    double wt[THREADS / 32];
};

// Merge every thread's (m, z, t) -- z, t relative to that thread's own m -- into the
// group's state relative to the group maximum.  `empty` threads contribute nothing.
// The result is valid in every thread.  Synchronises the group: call uniformly.
template <int THREADS, int BAR = 0>
__device__ __forceinline__ RowPartial block_merge(float m, double z, double t, bool empty,
                                                  ReduceSmem<THREADS>& sm) {
    constexpr int NW = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float mm = empty ? -INFINITY : m;
    float wm = warp_max_nan(mm);
    if (lane == 0) sm.wmax[warp] = wm;
    group_sync<THREADS, BAR>();
    float M = sm.wmax[0];
#pragma unroll
    for (int i = 1; i < NW; ++i) M = fmax_nan(M, sm.wmax[i]);
    double zc = 0.0, tc = 0.0;
    if (!empty) {
        float dm = m - M;  // <= 0, NaN if M or m is NaN
        float s = (dm == 0.f) ? 1.f : ex2(dm * kLog2e);
        zc = (double)s * z;
        tc = (double)s * (t + (double)dm * z);
    }
    zc = warp_sum(zc);
    tc = warp_sum(tc);
    if (lane == 0) {
        sm.wz[warp] = zc;
        sm.wt[warp] = tc;
    }
    group_sync<THREADS, BAR>();
    RowPartial r;
    r.z = 0.0;
    r.t = 0.0;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        r.z += sm.wz[i];
        r.t += sm.wt[i];
    }
    r.m = M;  // NaN poisons; -inf means every thread was empty
    if (M == -INFINITY) {
        r.z = 0.0;
        r.t = 0.0;
    }
    r.pad = 0.f;
    group_sync<THREADS, BAR>();  // smem is reused by the caller's next reduction
    return r;
}

// Merge two row partials (associative; fp64).  The reference's combine rule
// (csrc/fused_logprob.cu:119-154) with the -inf sentinel, evaluated in fp64.
__device__ __forceinline__ RowPartial merge_partials(RowPartial a, RowPartial b) {
    if (isnan(a.m) || isnan(b.m)) {
        RowPartial r = a;
        r.m = __int_as_float(0x7fc00000);
        return r;
    }
    if (b.m == -INFINITY) return a;
    if (a.m == -INFINITY) return b;
    float M = fmaxf(a.m, b.m);
    double da = (double)a.m - (double)M, db = (double)b.m - (double)M;
    double sa = exp(da), sb = exp(db);
    RowPartial r;
    r.m = M;
    r.z = sa * a.z + sb * b.z;
    r.t = sa * (a.t + da * a.z) + sb * (b.t + db * b.z);
    r.pad = 0.f;
    return r;
}

// Final per-row values from a merged partial and the target logit.
__device__ __forceinline__ void finalize_row(RowPartial p, double x_t, float* logprob,
                                             float* entropy, float* lse) {
    double l, h, lp;
    if (isnan(p.m)) {
        l = h = lp = (double)__int_as_float(0x7fc00000);
    } else if (p.m == -INFINITY) {
        l = -INFINITY;
        h = (double)__int_as_float(0x7fc00000);
        lp = x_t - l;
    } else {
        double logz = log(p.z);
        l = (double)p.m + logz;
        h = logz - p.t / p.z;
        lp = x_t - l;
    }
    *logprob = (float)lp;
    *entropy = (float)h;
    *lse = (float)l;
}

// ---------------------------------------------------------------------------------
// Row addressing (two stride levels, see include/k1_logprob.h)
// ---------------------------------------------------------------------------------
struct RowLayout {
    int64_t inner_rows;
    int64_t inner_stride;
    int64_t outer_stride;
    __device__ __forceinline__ int64_t offset(int64_t r) const {
        int64_t o = r / inner_rows;
        return o * outer_stride + (r - o * inner_rows) * inner_stride;
    }
};

}  // namespace k1
