// k1_lmhead.cuh -- the LM head fused with K1 on B200 tensor cores (tcgen05 + TMEM + TMA).
//
// Computes the logits z = bf16(h W^T) of an LM head tile by tile on the 5th-generation
// tensor cores and folds every tile into K1 in its epilogue, so the forward never writes
// the [N, V] logits to HBM:
//   STATS  per-row (m, Z, T) partials of the K1 forward over y = bf16(z * s) (s = 1/T, the
//          sampling temperature folded in with the rounding of `logits.div_(T)`), plus the
//          target logit; a small merge kernel turns them into (logprob, entropy, lse);
//   STORE  the same, and z itself is written (the training path that keeps the logits
//          for its backward);
//   GRAD   the K1 backward recomputed from the tile: dz = bf16(bf16(dL/dy) * s), written
//          in place of the logits (the memory-light training path's backward).
// The per-element arithmetic of the epilogues is K1's own (fwd_chunk, bwd_vector), applied
// to the bf16-rounded tile, so z, dz and the statistics are those of K1 on these logits.
//
// Kernel layout (one CTA per SM, persistent, 6 warps).  The default variant runs CTA
// pairs (a cluster of 2 CTAs on 2 SMs, tcgen05.mma.cta_group::2): each pair computes a
// 256 x 256 tile of the logits, each CTA holding its 128 rows of h and 128 rows of W per
// K block and its 128 x 256 half of the accumulator; the single-CTA variant (K1_LMH_PAIR=0)
// computes 128 x 256 tiles alone.
//   warp 0   TMA producer: 2-D tiled bulk-tensor copies (128-byte swizzle; every copy
//            reads this GPU's own memory into this CTA's own shared memory) of K blocks
//            of h and W into a ring (pair: 3 stages of 64 KB, each two 64-wide K
//            sub-blocks; single: 4 stages of 48 KB, one 64-wide K block), completion
//            counted on the pair leader's mbarrier;
//   warp 1   MMA issuer (the pair's first CTA): per 64-wide K sub-block, four tcgen05.mma
//            of kind::f16 (bf16 x bf16 -> fp32, K = 16 each) from shared memory into one
//            of two 256-column TMEM accumulators; tcgen05.commit releases the stage in
//            both CTAs and, after the last K block, hands the accumulator to both
//            epilogues.  A pair stage carries 1024 cycles of tensor work, twice the cost
//            of the stage's handshake (empty -> copies -> full -> MMAs -> commit), so the
//            handshakes stay off the tensor pipe's critical path;
//   warps 2-5  epilogue: each thread owns one row of its CTA's half tile (TMEM lane = row)
//            and reads its 256 fp32 accumulators 32 columns per wait with tcgen05.ld
//            (32x32b.x32), while the tensor cores fill the other accumulator.
// Work is cut into units of (a tile's rows, a run of consecutive 256-column tiles); the
// epilogue keeps each row's K1 state in registers across the unit's tiles and writes one
// partial per row and unit.  Units are ordered in groups of 16 row blocks, row block
// fastest, so the CTAs running at one time share a few W tiles and one group of h rows in
// L2 and W is read from HBM about once per group.
//
// Every mbarrier wait is bounded (ring::wait, a few seconds at most); a wait that runs out
// sets bit 3 of k1_ring_error and the CTA stops: the MMA thread waits (bounded) for its
// issued MMAs, the producer for its issued copies, and the TMEM is freed before exit.
#pragma once

#include <cuda.h>

#include "k1_ring.cuh"

namespace k1 {
namespace lmh {

constexpr int BM = 128;               // rows per tile (TMEM lanes)
constexpr int BN = 256;               // columns per tile (TMEM columns per accumulator)
constexpr int BK = 64;                // K per stage: 64 bf16 = one 128-byte swizzle row
constexpr int UK = 16;                // K per tcgen05.mma (kind::f16)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;  // 512: all of TMEM, so one CTA per SM
constexpr int EPI_WARPS = 4;
constexpr int THREADS = (2 + EPI_WARPS) * 32;
#ifndef K1_LMH_CW
#define K1_LMH_CW 32  // epilogue columns per TMEM wait: 32 or 64
#endif
static_assert(K1_LMH_CW == 32 || K1_LMH_CW == 64, "32 or 64 columns per epilogue step");
#ifndef K1_LMH_PREFETCH
#define K1_LMH_PREFETCH 0  // 1: prefetch the next tile's W into L2 while loading this one
#endif
#ifndef K1_LMH_GROUP_M
#define K1_LMH_GROUP_M 16
#endif
constexpr int GROUP_M = K1_LMH_GROUP_M;  // row blocks per L2 group

// tcgen05 instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B bf16 (bits
// 7-9 and 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at
// bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

enum Mode : int { STATS = 0, STORE = 1, GRAD = 2 };

struct Params {
    int64_t n_rows, vocab;  // vocab: the columns of this weight (a shard of the vocabulary)
    int64_t col_offset;     // global id of the weight's first row (vocab-parallel shards; else 0)
    int k_blocks;     // ceil(hidden / K per stage); copies beyond `hidden` read zeros
    int m_blocks;     // ceil(n_rows / BM)
    int n_tiles;      // ceil(vocab / BN)
    int n_parts;      // units per row block
    int units;        // m_blocks * n_parts
    float scale;      // y = bf16(z * scale) when SCALED
    const int64_t* targets;
    RowPartial* part;  // [n_parts][n_rows] (STATS, STORE)
    float* xt;         // [n_rows]: the target logit, written by the unit holding it
    // GRAD inputs (per row)
    const float* lse;
    const float* entropy;
    const float* g_logp;
    const float* g_ent;
    const float* g_lse;
    __nv_bfloat16* out;  // STORE: z; GRAD: dz; [n_rows] rows of out_stride elements
    int64_t out_stride;
    unsigned* done;      // STATS / STORE: epilogue warps that finished a unit (zeroed per launch)
};

// ------------------------------------------------------------------------------------
// PTX wrappers
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(ring::saddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(ring::saddr(bar))
        : "memory");
}

// Ask L2 to fetch a tile of the tensor (nothing lands in shared memory).
__device__ __forceinline__ void tma_prefetch_l2(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle: start address
// >> 4 (bits 0-13), leading offset unused (0), stride between 8-row groups 1024 B >> 4
// (bits 32-45), descriptor version 1 (bits 46-47), layout 2 = 128-byte swizzle (61-63).
// The tile must start on a 1024-byte boundary; the k-th 16-element slice of the 64-element
// swizzle row starts 32 k bytes further.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kIdesc), "r"(acc));
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                     "r"(ring::saddr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp-collective); the values
// may be read only after tmem_wait().
template <int OFF, int N>
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[N]) {
    static_assert(OFF + 32 <= N, "destination too small");
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[OFF + 0]), "=r"(r[OFF + 1]), "=r"(r[OFF + 2]), "=r"(r[OFF + 3]), "=r"(r[OFF + 4]),
          "=r"(r[OFF + 5]), "=r"(r[OFF + 6]), "=r"(r[OFF + 7]), "=r"(r[OFF + 8]), "=r"(r[OFF + 9]),
          "=r"(r[OFF + 10]), "=r"(r[OFF + 11]), "=r"(r[OFF + 12]), "=r"(r[OFF + 13]),
          "=r"(r[OFF + 14]), "=r"(r[OFF + 15]), "=r"(r[OFF + 16]), "=r"(r[OFF + 17]),
          "=r"(r[OFF + 18]), "=r"(r[OFF + 19]), "=r"(r[OFF + 20]), "=r"(r[OFF + 21]),
          "=r"(r[OFF + 22]), "=r"(r[OFF + 23]), "=r"(r[OFF + 24]), "=r"(r[OFF + 25]),
          "=r"(r[OFF + 26]), "=r"(r[OFF + 27]), "=r"(r[OFF + 28]), "=r"(r[OFF + 29]),
          "=r"(r[OFF + 30]), "=r"(r[OFF + 31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp-collective).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------------------------------
// Work decomposition
// ------------------------------------------------------------------------------------
struct Unit {
    int m_blk, part, n0, n1;  // row block, part index, tiles [n0, n1)
};

__device__ __forceinline__ Unit unit_of(const Params& p, int u) {
    const int per_group = GROUP_M * p.n_parts;
    const int g = u / per_group, r = u - g * per_group;
    const int rows_in_group = min(GROUP_M, p.m_blocks - g * GROUP_M);
    Unit x;
    x.part = r / rows_in_group;
    x.m_blk = g * GROUP_M + (r - x.part * rows_in_group);
    x.n0 = (int)((int64_t)x.part * p.n_tiles / p.n_parts);
    x.n1 = (int)((int64_t)(x.part + 1) * p.n_tiles / p.n_parts);
    return x;
}

// Bounded wait; on a timeout sets bit 3 of k1_ring_error and the CTA's abort flag.
__device__ __forceinline__ bool lmh_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    for (int i = 0; i < ring::kMaxTries; ++i) {
        if (ring::try_wait(bar, parity)) return true;
        if (*abort) return false;
    }
    atomicOr(&k1_ring_error, 8u);
    *abort = 1;
    return false;
}

// ------------------------------------------------------------------------------------
// Epilogue helpers
// ------------------------------------------------------------------------------------
// Round CW fp32 accumulators to bf16 pairs (the LM head's bf16 logits), columns at or
// beyond `valid` replaced by the vector padding (lowest finite bf16: e = 0).
template <int CW>
__device__ __forceinline__ void pack_tile_chunk(const uint32_t (&r)[CW], int valid,
                                                uint4 (&v)[CW / 8]) {
    uint32_t w[CW / 2];
#pragma unroll
    for (int i = 0; i < CW / 2; ++i)
        w[i] = DT<__nv_bfloat16>::from_f2(
            make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])));
    if (valid < CW) {  // the vocabulary's last chunk only
#pragma unroll
        for (int i = 0; i < CW / 2; ++i) {
            if (2 * i + 1 >= valid) w[i] = (w[i] & 0x0000FFFFu) | 0xFF7F0000u;
            if (2 * i >= valid) w[i] = DT<__nv_bfloat16>::kPadWord;
        }
    }
#pragma unroll
    for (int u = 0; u < CW / 8; ++u)
        v[u] = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
}

// Element k (0..CW-1) of a packed chunk as fp32.  k is known only at run time: one
// compare-and-select per word, every register named statically, so the chunk never goes
// through local memory (whose L1 traffic would compete with the tensor cores' operand
// reads from shared memory).
template <int NV>
__device__ __forceinline__ float chunk_elem(const uint4 (&v)[NV], int k) {
    const int j = k >> 1;
    uint32_t w = 0;
#pragma unroll
    for (int u = 0; u < NV; ++u) {
        w = j == 4 * u + 0 ? v[u].x : w;
        w = j == 4 * u + 1 ? v[u].y : w;
        w = j == 4 * u + 2 ? v[u].z : w;
        w = j == 4 * u + 3 ? v[u].w : w;
    }
    return (k & 1) ? __uint_as_float(w & 0xFFFF0000u) : __uint_as_float(w << 16);
}

// The temperature scale applied to a packed chunk, padding (columns >= valid) left as is
// (a scaled padding could overflow to -inf).
template <int NV>
__device__ __forceinline__ void scale_chunk(uint4 (&v)[NV], int valid, float s) {
    if (valid == NV * 8) {
#pragma unroll
        for (int k = 0; k < NV; ++k) v[k] = scale_vec<__nv_bfloat16>(v[k], s);
        return;
    }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const uint4 x = scale_vec<__nv_bfloat16>(v[k], s);
        const int b = k * 8;
        auto keep = [&](uint32_t scaled, uint32_t orig, int c) -> uint32_t {
            if (c + 1 >= valid) scaled = (scaled & 0x0000FFFFu) | (orig & 0xFFFF0000u);
            if (c >= valid) scaled = orig;
            return scaled;
        };
        v[k] = make_uint4(keep(x.x, v[k].x, b), keep(x.y, v[k].y, b + 2), keep(x.z, v[k].z, b + 4),
                          keep(x.w, v[k].w, b + 6));
    }
}

// Element k (0..CW-1) of a packed chunk replaced by bf16(val), with the same statically
// named selects as chunk_elem.
template <int NV>
__device__ __forceinline__ void set_chunk_elem(uint4 (&v)[NV], int k, float val) {
    const int j = k >> 1;
    const uint32_t b = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(val));
    const uint32_t keep = (k & 1) ? 0x0000FFFFu : 0xFFFF0000u;
    const uint32_t put = (k & 1) ? (b << 16) : b;
#pragma unroll
    for (int u = 0; u < NV; ++u) {
        v[u].x = j == 4 * u + 0 ? ((v[u].x & keep) | put) : v[u].x;
        v[u].y = j == 4 * u + 1 ? ((v[u].y & keep) | put) : v[u].y;
        v[u].z = j == 4 * u + 2 ? ((v[u].z & keep) | put) : v[u].z;
        v[u].w = j == 4 * u + 3 ? ((v[u].w & keep) | put) : v[u].w;
    }
}

// Store the first `valid` bf16 columns of a packed chunk of one row (the ragged or
// unaligned case element by element, every register named statically).
// 32 bytes at a 32-byte aligned address in one store.
__device__ __forceinline__ void stg32(void* p, uint4 a, uint4 b) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a.x),
                 "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                 : "memory");
}

// vec: 16-byte aligned row pieces (16-byte stores); vec32: 32-byte aligned (32-byte stores,
// half the store instructions, each touching the warp's 32 rows once).
template <int NV>
__device__ __forceinline__ void store_chunk(__nv_bfloat16* dst, const uint4 (&v)[NV], int valid,
                                            bool vec_ok, bool vec32_ok = false) {
    if (vec32_ok && valid >= NV * 8 && NV % 2 == 0) {
#pragma unroll
        for (int u = 0; u < NV; u += 2) stg32(reinterpret_cast<uint4*>(dst) + u, v[u], v[u + 1]);
    } else if (vec_ok && valid >= NV * 8) {
        uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int u = 0; u < NV; ++u) stg_stream(d + u, v[u]);
    } else {
        unsigned short* d = reinterpret_cast<unsigned short*>(dst);
#pragma unroll
        for (int u = 0; u < NV; ++u) {
            const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = u * 8 + 2 * i;
                if (c < valid) d[c] = (unsigned short)(w[i] & 0xFFFFu);
                if (c + 1 < valid) d[c + 1] = (unsigned short)(w[i] >> 16);
            }
        }
    }
}

// Geometry of the two variants.  PAIR = false: one CTA computes a 128 x 256 tile with
// tcgen05.mma.cta_group::1 (M = 128) from a 4-stage ring of 48 KB (its 128 rows of h and
// 256 rows of W per K block).  PAIR = true: a cluster of two CTAs on two SMs computes a
// 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256) issued by the first CTA; each
// CTA holds its 128 rows of h and its 128 rows of W per K block (32 KB; 6 stages), its
// own 128 x 256 half of the accumulator in its own TMEM, and runs its own epilogue.  The
// pair moves half the bytes per flop through shared memory and L2 of the single CTA.
#ifndef K1_LMH_PAIR_KSUB
#define K1_LMH_PAIR_KSUB 2  // 64-wide K sub-blocks per pair stage: 1 or 2
#endif
#ifndef K1_LMH_PAIR_STAGES
#define K1_LMH_PAIR_STAGES (K1_LMH_PAIR_KSUB == 2 ? 3 : 6)
#endif
static_assert(K1_LMH_PAIR_KSUB == 1 || K1_LMH_PAIR_KSUB == 2, "1 or 2 K sub-blocks per stage");
template <bool PAIR>
struct Geo {
    static constexpr int CTAS = PAIR ? 2 : 1;
    static constexpr int TILE_M = BM * CTAS;        // rows per tile (all CTAs of the pair)
    static constexpr int LOAD_N = BN / CTAS;        // W rows per CTA and K block
    static constexpr int KSUB = PAIR ? K1_LMH_PAIR_KSUB : 1;  // 64-wide K sub-blocks per stage
    static constexpr int KB = BK * KSUB;            // K per stage
    static constexpr int A_SUB = BM * BK * 2;       // 16 KB: one swizzled 128 x 64 box of h
    static constexpr int B_SUB = LOAD_N * BK * 2;   // 32 KB alone, 16 KB in a pair
    static constexpr int A_B = KSUB * A_SUB;
    static constexpr int B_B = KSUB * B_SUB;
    static constexpr int STAGE_B = A_B + B_B;
    static constexpr int NSTAGE = PAIR ? K1_LMH_PAIR_STAGES : STAGES;
    static constexpr int SMEM = 1024 + NSTAGE * STAGE_B + 256;
    static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) |
                                      ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TILE_M >> 4) << 24);
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of `saddr` (a shared::cta address) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
// Every thread of both CTAs (per-thread form: the warps need not be converged).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (address from mapa).  The default
// (CTA-scope) semantics: a release at cluster scope here would make the arriving thread
// wait for its own bulk copies in flight, which serialises the producer.
__device__ __forceinline__ void arrive_remote(uint32_t cl_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
// Tiled 2-D copy into this CTA's shared memory whose completion is counted on the pair
// leader's mbarrier (cl_bar, a shared::cluster address).  Each CTA copies
// only its own tile, from this GPU's memory.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t cl_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(ring::saddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(cl_bar)
        : "memory");
}
template <bool PAIR>
__device__ __forceinline__ void umma_t(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc) {
    if constexpr (PAIR) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(da), "l"(db), "r"(Geo<true>::IDESC), "r"(acc));
    } else {
        umma(tmem_d, da, db, acc);
    }
}
// Arrive on `bar` (this CTA's, or in both CTAs of the pair) once this thread's issued
// tcgen05 operations have completed.
template <bool PAIR>
__device__ __forceinline__ void commit_t(uint64_t* bar) {
    if constexpr (PAIR) {
        const uint16_t both = 0x3;
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
            "[%0], %1;" ::"r"(ring::saddr(bar)),
            "h"(both)
            : "memory");
    } else {
        umma_commit(bar);
    }
}

template <int MODE, bool SCALED, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    k1_lmhead_kernel(const __grid_constant__ CUtensorMap tmap_h,
                     const __grid_constant__ CUtensorMap tmap_w, Params p) {
    using GE = Geo<PAIR>;
    constexpr int NST = GE::NSTAGE;
    extern __shared__ __align__(16) unsigned char lmh_raw[];
    // 1024-byte aligned ring (128-byte swizzle atoms), barriers after it
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(lmh_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * GE::STAGE_B);
    uint64_t* empty = full + NST;
    uint64_t* tfull = empty + NST;
    uint64_t* tempty = tfull + NUM_ACC;
    uint64_t* drain = tempty + NUM_ACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;  // 0: the pair's MMA leader
    const bool leader = rank == 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            ring::bar_init(&full[s], GE::CTAS);  // both producers arrive at the leader's
            ring::bar_init(&empty[s], 1);
        }
        for (int a = 0; a < NUM_ACC; ++a) {
            ring::bar_init(&tfull[a], 1);
            ring::bar_init(&tempty[a], GE::CTAS * EPI_WARPS * 32);  // both epilogues
        }
        ring::bar_init(drain, 1);
        *abort = 0;
        ring::fence_init();
    }
    if (warp == 0) {
        prefetch_tmap(&tmap_h);
        prefetch_tmap(&tmap_w);
    }
    if (warp == 1) {  // all of this SM's TMEM (one CTA per SM); in a pair, both CTAs' warps
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             ring::saddr(tmem_slot)),
                         "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             ring::saddr(tmem_slot)),
                         "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    __syncwarp();
    tc_fence_before();
    if constexpr (PAIR)
        cluster_sync();  // the peer's barriers are initialised before any remote arrival
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int G = gridDim.x / GE::CTAS;        // CTAs (pairs) in the grid
    const int me = blockIdx.x / GE::CTAS;      // this CTA's (pair's) index

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (int u = me; ok && u < p.units; u += G) {
                const Unit x = unit_of(p, u);
                for (int n = x.n0; ok && n < x.n1; ++n) {
                    for (int kb = 0; kb < p.k_blocks; ++kb) {
                        if (!lmh_wait(&empty[stage], phase ^ 1u, abort)) {
                            ok = false;
                            break;
                        }
#ifdef K1_WAIT_TEST
                        if (blockIdx.x == 0 && (long long)issued == k1_test_withhold) {
                            ok = false;  // test-only: CTA 0 issues nothing more
                            break;
                        }
#endif
                        unsigned char* sa = smem + stage * GE::STAGE_B;
                        const int row_a = x.m_blk * GE::TILE_M + (int)rank * BM;
                        const int row_b = n * BN + (int)rank * GE::LOAD_N;
                        if constexpr (PAIR) {
                            const uint32_t cl = mapa(ring::saddr(&full[stage]), 0);
#pragma unroll
                            for (int j = 0; j < GE::KSUB; ++j)
                                tma_load_2d_pair(sa + j * GE::A_SUB, &tmap_h, kb * GE::KB + j * BK, row_a, cl);
#pragma unroll
                            for (int j = 0; j < GE::KSUB; ++j)
                                tma_load_2d_pair(sa + GE::A_B + j * GE::B_SUB, &tmap_w, kb * GE::KB + j * BK,
                                                 row_b, cl);
                            if (leader)
                                ring::arrive_expect(&full[stage], GE::CTAS * GE::STAGE_B);
                            else
                                arrive_remote(cl);
                        } else {
                            ring::arrive_expect(&full[stage], GE::STAGE_B);
                            tma_load_2d(sa, &tmap_h, kb * BK, row_a, &full[stage]);
                            tma_load_2d(sa + GE::A_B, &tmap_w, kb * BK, row_b, &full[stage]);
                        }
                        // the next tile's W rows of this K block into L2, a tile ahead
                        if (K1_LMH_PREFETCH && n + 1 < x.n1)
                            for (int j = 0; j < GE::KSUB; ++j)
                                tma_prefetch_l2(&tmap_w, kb * GE::KB + j * BK, row_b + BN);
                        ++issued;
                        if (++stage == NST) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (!ok && leader) {
                // stopping early: wait (bounded) for the copies still in flight
                for (uint32_t i = (issued > NST ? issued - NST : 0u); i < issued; ++i)
                    ring::wait(&full[i % NST], (i / NST) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (the pair's leader) ----------------
        if (lane == 0 && leader) {
            uint32_t stage = 0, phase = 0;
            int t = 0;  // tiles so far
            bool ok = true;
            const uint32_t sbase = ring::saddr(smem);
            for (int u = me; ok && u < p.units; u += G) {
                const Unit x = unit_of(p, u);
                for (int n = x.n0; ok && n < x.n1; ++n, ++t) {
                    const int a = t & 1;
                    if (!lmh_wait(&tempty[a], ((t >> 1) & 1) ^ 1u, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(a * BN);
                    for (int kb = 0; kb < p.k_blocks; ++kb) {
                        if (!lmh_wait(&full[stage], phase, abort)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = sbase + stage * GE::STAGE_B;
#pragma unroll
                        for (int j = 0; j < GE::KSUB; ++j) {
                            const uint64_t da = smem_desc(sa + j * GE::A_SUB);
                            const uint64_t db = smem_desc(sa + GE::A_B + j * GE::B_SUB);
#pragma unroll
                            for (int k = 0; k < BK / UK; ++k)  // +32 bytes per K slice: +2 in >> 4 units
                                umma_t<PAIR>(d, da + 2 * k, db + 2 * k, (kb > 0 || j > 0 || k > 0) ? 1u : 0u);
                        }
                        commit_t<PAIR>(&empty[stage]);  // the stage is free once these MMAs ran
                        if (++stage == NST) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (ok) commit_t<PAIR>(&tfull[a]);  // the accumulator is complete
                }
            }
            // every MMA issued has completed before the TMEM can be freed
            commit_t<PAIR>(drain);
            ring::wait(drain, 0);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;  // TMEM lanes 32 quarter .. 32 quarter + 31
        const int rloc = quarter * 32 + lane;
        const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16);
        const bool vec_ok = (p.out_stride & 7) == 0 &&
                            (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
        const bool vec32_ok = (p.out_stride & 15) == 0 &&
                              (reinterpret_cast<uintptr_t>(p.out) & 31) == 0;
        int t = 0;
        bool ok = true;
        int u_fail = -1, n_fail = 0;  // where a wait ran out
        for (int u = me; ok && u < p.units; u += G) {
            const Unit x = unit_of(p, u);
            const int64_t row = (int64_t)x.m_blk * GE::TILE_M + (int64_t)rank * BM + rloc;
            const bool live = row < p.n_rows;
            const int64_t tg = live ? p.targets[row] : -1;  // a global token id
            const int64_t tt = tg - p.col_offset;
            const int64_t tcol = (tg >= 0 && tt >= 0 && tt < p.vocab) ? tt : -1;
            FwdState st;
            st.init();
            float xt = 0.f;
            bool has_xt = false;
            BwdRow q;
            if constexpr (MODE == GRAD) {
                q.lse = live ? p.lse[row] : 0.f;
                q.ent = live ? p.entropy[row] : 0.f;
                q.gl = (live && p.g_logp) ? p.g_logp[row] : 0.f;
                q.ge = (live && p.g_ent) ? p.g_ent[row] : 0.f;
                q.gs = (live && p.g_lse) ? p.g_lse[row] : 0.f;
                q.c0 = q.gs - q.gl - q.ge * q.ent;
                q.tl = tcol;
            }
            for (int n = x.n0; n < x.n1; ++n, ++t) {
                const int a = t & 1;
                // warp-uniform: the TMEM loads below are warp-collective
                if (!__all_sync(0xffffffffu, lmh_wait(&tfull[a], (t >> 1) & 1, abort))) {
                    ok = false;
                    u_fail = u;
                    n_fail = n;
                    break;
                }
                tc_fence_after();
                constexpr int CW = K1_LMH_CW;  // columns per step, 32 per TMEM load, one wait
                for (int c = 0; c < BN / CW; ++c) {
                    uint32_t r[CW];
                    __syncwarp();  // converged for the warp-collective TMEM loads
                    tmem_ld32_async<0>(tlane + (uint32_t)(a * BN + c * CW), r);
                    if constexpr (CW == 64)
                        tmem_ld32_async<32 % CW>(tlane + (uint32_t)(a * BN + c * CW + 32), r);
                    tmem_wait();
                    const int64_t col0 = (int64_t)n * BN + c * CW;
                    const int64_t left = p.vocab - col0;
                    const int valid = left < CW ? (int)left : CW;
                    if (valid <= 0) continue;
                    uint4 v[CW / 8];
                    pack_tile_chunk<CW>(r, valid, v);
                    __nv_bfloat16* dst = p.out + row * p.out_stride + col0;
                    if constexpr (MODE == GRAD) {
                        uint4 o[CW / 8];
#pragma unroll
                        for (int k = 0; k < CW / 8; ++k) o[k] = bwd_vector<__nv_bfloat16, SCALED>(v[k], q, p.scale);
                        if (tcol >= col0 && tcol < col0 + CW) {
                            const int k = (int)(tcol - col0);
                            float y = chunk_elem(v, k);
                            if (SCALED) y = scale1<__nv_bfloat16>(y, p.scale);
                            const float g = scale1<__nv_bfloat16>(
                                DT<__nv_bfloat16>::round1(bwd_target_value(y, q)), p.scale);
                            set_chunk_elem(o, k, g);
                        }
                        if (live) store_chunk(dst, o, valid, vec_ok, vec32_ok);
                    } else {
                        if constexpr (MODE == STORE) {
                            if (live) store_chunk(dst, v, valid, vec_ok, vec32_ok);
                        }
                        if constexpr (SCALED) scale_chunk(v, valid, p.scale);
                        if (tcol >= col0 && tcol < col0 + CW) {
                            xt = chunk_elem(v, (int)(tcol - col0));
                            has_xt = true;
                        }
                        fwd_chunk<__nv_bfloat16, CW / 8>(v, st, false);
                    }
                }
                tc_fence_before();
                if constexpr (PAIR) {
                    if (leader)
                        ring::arrive(&tempty[a]);
                    else
                        arrive_remote(mapa(ring::saddr(&tempty[a]), 0));
                } else {
                    ring::arrive(&tempty[a]);
                }
            }
            if (!ok) break;
            if constexpr (MODE != GRAD) {
                if (live) {
                    RowPartial o;
                    const bool empty_state = st.m <= DT<__nv_bfloat16>::kLowest;
                    o.m = empty_state ? -INFINITY : st.m;
                    o.z = empty_state ? 0.0 : st.z64();
                    o.t = empty_state ? 0.0 : st.t64();
                    o.pad = 0.f;
                    p.part[(int64_t)x.part * p.n_rows + row] = o;
                    if (has_xt) p.xt[row] = xt;
                }
                // count this warp's rows of the unit in: the merge kernel turns a launch
                // with a missing unit (a wait that ran out) into NaN outputs
                __syncwarp();
                if (lane == 0) {
                    __threadfence();
                    atomicAdd(p.done, 1u);
                }
            }
        }
        if constexpr (MODE == GRAD) {
            // a wait ran out: the gradient tiles this thread did not write become NaN
            if (u_fail >= 0) {
                const uint32_t nw = DT<__nv_bfloat16>::kNaNWord;
                uint4 nanv[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) nanv[k] = make_uint4(nw, nw, nw, nw);
                for (int u = u_fail; u < p.units; u += G) {
                    const Unit x = unit_of(p, u);
                    const int64_t row = (int64_t)x.m_blk * GE::TILE_M + (int64_t)rank * BM + rloc;
                    if (row >= p.n_rows) continue;
                    for (int n = (u == u_fail ? n_fail : x.n0); n < x.n1; ++n) {
                        for (int c = 0; c < BN / 64; ++c) {
                            const int64_t col0 = (int64_t)n * BN + c * 64;
                            const int64_t left = p.vocab - col0;
                            if (left <= 0) break;
                            store_chunk(p.out + row * p.out_stride + col0, nanv,
                                        left < 64 ? (int)left : 64, vec_ok);
                        }
                    }
                }
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    if constexpr (PAIR)
        cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals may touch it
    else
        __syncthreads();
    tc_fence_after();
    __syncwarp();
    if (warp == 1) {
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                         "r"(TMEM_COLS)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                         "r"(TMEM_COLS)
                         : "memory");
    }
}

// Vocab-parallel shard: the same merge, written as the row's k1_partial (relative to the
// shard's maximum; the target logit when the target's column lies in the shard) for the
// all-gather and k1_vocab_combine.  A launch with a missing unit gives NaN partials.
__global__ void k1_lmhead_shard_merge_kernel(const RowPartial* part, const float* xt,
                                             const int64_t* targets, int64_t n_rows,
                                             int64_t vocab, int64_t col_offset, int n_parts,
                                             const unsigned* done, unsigned expected,
                                             k1_partial* out) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= n_rows) return;
    k1_partial o;
    o.reserved = 0;
    if (*done != expected) {
        const float nan = __int_as_float(0x7fc00000);
        o.z = o.t = (double)nan;
        o.m = o.x_t = nan;
        o.has_target = 0;
        out[row] = o;
        return;
    }
    RowPartial acc;
    acc.m = -INFINITY;
    acc.z = acc.t = 0.0;
    acc.pad = 0.f;
    for (int i = 0; i < n_parts; ++i) acc = merge_partials(acc, part[(int64_t)i * n_rows + row]);
    const int64_t tg = targets[row], tt = tg - col_offset;
    const bool has = tg >= 0 && tt >= 0 && tt < vocab;
    o.m = acc.m;
    o.z = acc.m == -INFINITY ? 0.0 : acc.z;
    o.t = acc.m == -INFINITY ? 0.0 : acc.t;
    o.x_t = has ? xt[row] : 0.f;
    o.has_target = has ? 1 : 0;
    out[row] = o;
}

// Merge the units' partials of every row (fp64, in part order) and finish the row.
// A launch that did not finish every unit (a bounded wait ran out) gives NaN for all rows.
__global__ void k1_lmhead_merge_kernel(const RowPartial* part, const float* xt,
                                       const int64_t* targets, int64_t n_rows, int64_t vocab,
                                       int n_parts, const unsigned* done, unsigned expected,
                                       float* logprob, float* entropy, float* lse) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= n_rows) return;
    if (*done != expected) {
        const float nan = __int_as_float(0x7fc00000);
        logprob[row] = entropy[row] = lse[row] = nan;
        return;
    }
    RowPartial acc;
    acc.m = -INFINITY;
    acc.z = acc.t = 0.0;
    acc.pad = 0.f;
    for (int i = 0; i < n_parts; ++i) acc = merge_partials(acc, part[(int64_t)i * n_rows + row]);
    const int64_t tg = targets[row];
    const double x = (tg >= 0 && tg < vocab) ? (double)xt[row] : 0.0;
    finalize_row(acc, x, logprob + row, entropy + row, lse + row);
}

}  // namespace lmh
}  // namespace k1
