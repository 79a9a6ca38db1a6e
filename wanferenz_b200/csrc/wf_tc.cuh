// wf_tc.cuh - tcgen05 (5th-generation tensor core) building blocks for sm_100a:
// TMEM allocation, block-scaled MMA (kind::mxf8f6f4.block_scale), tensor-memory
// loads/stores, commit-to-mbarrier, 2D tiled TMA loads, and the shared-memory
// matrix / instruction descriptors.
//
// Operand conventions used by the kernels:
//   A = weight rows (M = 128 per MMA), K-major, 128-byte swizzled rows in
//       shared memory, loaded by TMA: E2M1 through the unpacking tensor-map
//       type 16U4_ALIGN16B (16 packed nibbles + 8 zero bytes per 16-byte
//       chunk, 1 byte per element on average), E4M3 as plain bytes;
//   B = tokens (N = 16 or 32 per MMA), E4M3, K-major, same swizzle, written by
//       the worker warps after quantizing activations;
//   D = f32 accumulator in TMEM: lane = weight row, column = token;
//   scale factors (UE8M0, one per 32 K) in TMEM, 4 consecutive K-blocks of one
//       row packed in one 32-bit column word; for 128 rows the word of row
//       r = r0 + 32*r1 sits at lane r0 (replicated in all 4 lane quadrants),
//       column base + r1.  The MMA picks the byte with the descriptor's sf_id.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "wf_ptx.cuh"

namespace wf {
namespace tc {

// ---- TMEM allocation (one warp) -----------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// ---- ordering of tcgen05 operations around thread synchronization ------
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- block-scaled MMA: D[tmem] (+)= A[smem] x B[smem], scales in TMEM ----
__device__ __forceinline__ void mma_mxf8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far is complete.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// ---- TMEM <-> registers (a warp accesses the 32 lanes of its quadrant) --
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c,
                                         uint32_t d) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr),
                 "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- 2D tiled TMA load, completion on an mbarrier -----------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// 3D tiled TMA load, completion on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// L2 policy for streamed weights: evict first, so a layer step's ~1 GB of weights
// passing through the 126 MB L2 does not displace the kernels' instructions, the
// routing tables and the activations, which are read again.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// tma_load_2d / tma_load_3d with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar,
                                                 uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                                 uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Prefetch one 2D box of the tensor map into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *map, int c0, int c1) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1)
                 : "memory");
}

// ---- descriptors -------------------------------------------------------------
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes (SBO), start address in 16-byte units, descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *p) {
    const uint64_t addr = (smem_u32(p) & 0x3ffffu) >> 4;
    uint64_t d = 0;
    d |= addr;                       // [0,14) start address
    d |= (uint64_t)1 << 16;          // [16,30) leading byte offset (16 B, unused for SW128 K-major)
    d |= (uint64_t)(1024 >> 4) << 32;  // [32,46) stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;          // [46,48) version
    d |= (uint64_t)2 << 61;          // [61,64) layout: 128-byte swizzle
    return d;
}

// Instruction descriptor of kind::mxf8f6f4.block_scale with UE8M0 scales,
// M = 128, dense, both operands K-major.
//   a_fmt / b_fmt: 0 = E4M3, 5 = E2M1.
__device__ __forceinline__ uint32_t idesc_mxf8f6f4(int a_fmt, int b_fmt, int n, int sf_id) {
    uint32_t d = 0;
    d |= (uint32_t)(sf_id & 3) << 4;   // B scale-factor byte
    d |= (uint32_t)(a_fmt & 7) << 7;
    d |= (uint32_t)(b_fmt & 7) << 10;
    d |= (uint32_t)((n >> 3) & 63) << 17;
    d |= 1u << 23;                     // scale format UE8M0
    d |= (uint32_t)((128 >> 4) & 31) << 24;
    d |= (uint32_t)(sf_id & 3) << 29;  // A scale-factor byte
    return d;
}

// Byte offset inside a 128-byte-swizzled K-major tile of the 16-byte chunk
// `chunk` (0..7) of row `row`.
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
    return (uint32_t)row * 128u + (uint32_t)((chunk ^ (row & 7)) << 4);
}

}  // namespace tc
}  // namespace wf

namespace wf {
namespace tc {

// ---------------------------------------------------------------------------
// Dense block-scaled skinny GEMM on tcgen05:
//   out[m, n] = sum_k (a[m,k] * sa[m,k/128]) * (w[n,k] * sw[n,k/32 or n/128,k/128])
// for <= 16 tokens per item (MMA N = 16), weight tiles of 128 rows (MMA M),
// K split into chunks of <= 4096 (split-K partials reduced by the last chunk).
// ---------------------------------------------------------------------------
constexpr int W_PROD = 0, W_MMA = 1, W_WORK0 = 2;  // warp roles; 4 worker warps
constexpr int THREADS = 6 * 32;
constexpr int STAGES = 8;
constexpr int ABOX = 128 * 128;          // shared bytes of one 128x128 A box
constexpr int NTOK = 16;                 // tokens per item (MMA N)
constexpr int BSTEP = NTOK * 128;        // shared bytes of one 128-wide K step of B
constexpr int KC_MAX = 4096;
constexpr int OFF_B = STAGES * ABOX;
constexpr int OFF_BAR = OFF_B + (KC_MAX / 128) * BSTEP;
constexpr int NBAR = 2 * STAGES + 10;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 64 + 1024;  // + alignment slack
// TMEM columns
constexpr uint32_t COL_D = 0;      // 2 x 32
constexpr uint32_t COL_SFB = 64;   // 128
constexpr uint32_t COL_SFA = 256;  // 2 x 128

struct DenseArgs {
    CUtensorMap tmA;  // weights, box 128 (K) x 128 (rows), 128-byte swizzle
    const uint8_t *a;     // e4m3 tokens [M, K]
    const uint8_t *a_s;   // e8m0 [M, K/128]
    const uint8_t *w_s;   // FP4: e8m0 [N, K/32]; FP8: e8m0 [N/128, K/128]
    int fp4, M, N, K, nkc, Kc;
    __nv_bfloat16 *out;   // [M, N]
    float *part;          // [nkc, M, N] (nkc > 1)
    unsigned *cnt;        // [ceil(M/16) * N/128 * 4] (nkc > 1)
    int *err;
};

struct DItem {
    int kc, tg, tile, tok0, ntok, key;
};

__device__ __forceinline__ DItem dense_item(const DenseArgs &d, int i) {
    const int ntile = d.N / 128, ntg = (d.M + NTOK - 1) / NTOK;
    DItem it;
    it.kc = i / (ntg * ntile);
    const int rem = i % (ntg * ntile);
    it.tg = rem / ntile;
    it.tile = rem % ntile;
    it.tok0 = it.tg * NTOK;
    it.ntok = min(NTOK, d.M - it.tok0);
    it.key = it.kc * ntg + it.tg;
    return it;
}

struct Bars {
    uint64_t *full, *empty, *b_ready, *b_free, *sfa_ready, *sfa_free, *d_ready, *d_free;
    uint32_t *tmem_base;
    volatile int *abort;
    int *last;
};

__device__ __forceinline__ Bars bars_at(uint8_t *base) {
    uint64_t *b = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    Bars r;
    r.full = b;
    r.empty = b + STAGES;
    r.b_ready = b + 2 * STAGES;
    r.b_free = b + 2 * STAGES + 1;
    r.sfa_ready = b + 2 * STAGES + 2;  // [2]
    r.sfa_free = b + 2 * STAGES + 4;   // [2]
    r.d_ready = b + 2 * STAGES + 6;    // [2]
    r.d_free = b + 2 * STAGES + 8;     // [2]
    r.tmem_base = reinterpret_cast<uint32_t *>(b + NBAR);
    r.abort = reinterpret_cast<volatile int *>(b + NBAR) + 1;
    r.last = reinterpret_cast<int *>(b + NBAR) + 2;
    return r;
}

__device__ __forceinline__ bool twait(uint64_t *bar, uint32_t parity, int *err, volatile int *abort) {
    if (*abort) return false;
    if (!wf_wait(bar, parity, err)) { *abort = 1; return false; }
    return true;
}

__global__ void __launch_bounds__(THREADS, 1) k_dense_tc(const __grid_constant__ DenseArgs d) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Bars B = bars_at(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Programmatic dependent launch: set-up and the first ring of weight loads
    // (constant data) overlap the previous kernel; every thread waits for it
    // before its first bounded wait, and the worker warps, which read the
    // activations and write every output, before anything else.
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(B.full + s, 1); mbar_init(B.empty + s, 1); }
        mbar_init(B.b_ready, 4);
        mbar_init(B.b_free, 1);
        for (int j = 0; j < 2; ++j) {
            mbar_init(B.sfa_ready + j, 4); mbar_init(B.sfa_free + j, 1);
            mbar_init(B.d_ready + j, 1); mbar_init(B.d_free + j, 4);
        }
        *B.abort = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) { tmem_alloc(B.tmem_base, 512); tmem_relinquish(); }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = *B.tmem_base;
    const int ntile = d.N / 128, ntg = (d.M + NTOK - 1) / NTOK;
    const int n = d.nkc * ntg * ntile;
    const int i0 = (int)(((long long)n * blockIdx.x) / gridDim.x);
    const int i1 = (int)(((long long)n * (blockIdx.x + 1)) / gridDim.x);
    const int nks = d.Kc / 128;  // K steps per item
    uint8_t *Bsm = base + OFF_B;

    if (warp == W_PROD) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int gs = 0;
            for (int i = i0; i < i1 && !*B.abort; ++i) {
                const DItem it = dense_item(d, i);
                for (int s = 0; s < nks; ++s, ++gs) {
                    const int st = gs % STAGES;
                    // the first ring of weight loads overlaps the previous kernel; no
                    // bounded wait starts before that kernel is complete
                    if (gs == STAGES) pdl_wait();
                    if (gs >= STAGES && !twait(B.empty + st, ((gs / STAGES) - 1) & 1, d.err, B.abort)) break;
                    mbar_arrive_expect_tx(B.full + st, d.fp4 ? ABOX / 2 : ABOX);
                    tma_load_2d_hint(base + st * ABOX, &d.tmA, it.kc * d.Kc + s * 128, it.tile * 128, B.full + st,
                                     pol);
                }
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            pdl_wait();
            int gs = 0, nb = 0, key = -1;
            const int afmt = d.fp4 ? 5 : 0;
            for (int q = 0, i = i0; i < i1 && !*B.abort; ++i, ++q) {
                const DItem it = dense_item(d, i);
                const int buf = q & 1;
                if (it.key != key) {
                    if (!twait(B.b_ready, nb & 1, d.err, B.abort)) break;
                    ++nb;
                    key = it.key;
                }
                if (!twait(B.sfa_ready + buf, (q >> 1) & 1, d.err, B.abort)) break;
                if (q >= 2 && !twait(B.d_free + buf, ((q >> 1) - 1) & 1, d.err, B.abort)) break;
                fence_after_sync();
                const uint32_t dcol = tm + COL_D + 32 * buf;
                for (int s = 0; s < nks; ++s, ++gs) {
                    const int st = gs % STAGES;
                    if (!twait(B.full + st, (gs / STAGES) & 1, d.err, B.abort)) break;
                    fence_after_sync();
                    const uint64_t ad = smem_desc_sw128(base + st * ABOX);
                    const uint64_t bd = smem_desc_sw128(Bsm + s * BSTEP);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        mma_mxf8f6f4(dcol, ad + 2 * j, bd + 2 * j, idesc_mxf8f6f4(afmt, 0, NTOK, j),
                                     tm + COL_SFA + 128 * buf + 4 * s, tm + COL_SFB + 4 * s,
                                     (s | j) != 0);
                    commit(B.empty + st);
                }
                commit(B.d_ready + buf);
                commit(B.sfa_free + buf);
                const bool last_of_set = (i + 1 >= i1) || dense_item(d, i + 1).key != it.key;
                if (last_of_set) commit(B.b_free);
            }
        }
    } else {
        // ---- worker warps: B operand, scale factors, epilogue ----
        pdl_wait();
        const int wq = warp & 3;          // TMEM lane quadrant of this warp
        const int wt = threadIdx.x - W_WORK0 * 32;  // 0..127
        const uint32_t lane_base = (uint32_t)(32 * wq) << 16;
        const int K = d.K, kb_all = K / 128;
        int nb = 0, key = -1;
        auto epilogue = [&](int qe, const DItem &ie) {
            const int buf = qe & 1;
            if (!twait(B.d_ready + buf, (qe >> 1) & 1, d.err, B.abort)) return;
            fence_after_sync();
            uint32_t v[16];
            tmem_ld16(tm + lane_base + COL_D + 32 * buf, v);
            tmem_wait_ld();
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(B.d_free + buf);
            const int row = ie.tile * 128 + 32 * wq + lane;
            if (d.nkc == 1) {
#pragma unroll
                for (int m = 0; m < NTOK; ++m)
                    if (m < ie.ntok)
                        d.out[(size_t)(ie.tok0 + m) * d.N + row] = __float2bfloat16_rn(__uint_as_float(v[m]));
            } else {
                // split-K: this warp's 32 rows; the last K chunk to arrive (per tile and
                // lane quadrant) sums the partials in chunk order
#pragma unroll
                for (int m = 0; m < NTOK; ++m)
                    if (m < ie.ntok)
                        d.part[((size_t)ie.kc * d.M + ie.tok0 + m) * d.N + row] = __uint_as_float(v[m]);
                __threadfence();
                __syncwarp();
                unsigned *cnt = d.cnt + ((size_t)ie.tg * ntile + ie.tile) * 4 + wq;
                int last = 0;
                if (lane == 0) last = atomicAdd(cnt, 1u) == (unsigned)d.nkc - 1;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    // chunk outer, tokens inner: the tokens' loads of one chunk are in
                    // flight together; each token's sum still runs in chunk order
                    float acc[NTOK];
#pragma unroll
                    for (int m = 0; m < NTOK; ++m) acc[m] = 0.f;
#pragma unroll 4
                    for (int c = 0; c < d.nkc; ++c) {
                        const float *pc = d.part + ((size_t)c * d.M + ie.tok0) * d.N + row;
                        float v[NTOK];
#pragma unroll
                        for (int m = 0; m < NTOK; ++m) v[m] = m < ie.ntok ? __ldcg(pc + (size_t)m * d.N) : 0.f;
#pragma unroll
                        for (int m = 0; m < NTOK; ++m) acc[m] += v[m];
                    }
#pragma unroll
                    for (int m = 0; m < NTOK; ++m)
                        if (m < ie.ntok) d.out[(size_t)(ie.tok0 + m) * d.N + row] = __float2bfloat16_rn(acc[m]);
                    if (lane == 0) *cnt = 0u;
                }
            }
        };
        DItem prev{};
        int qprev = -1;
        for (int q = 0, i = i0; i < i1; ++i, ++q) {
            if (*B.abort) break;
            const DItem it = dense_item(d, i);
            const int buf = q & 1;
            if (it.key != key) {
                // new token set: B tile (E4M3, swizzled) for the whole K chunk + its scales
                if (nb > 0 && !twait(B.b_free, (nb - 1) & 1, d.err, B.abort)) break;
                const int row = wt >> 3, chunk = wt & 7;
                const bool rv = row < it.ntok;
                const uint8_t *src = d.a + (size_t)(it.tok0 + (rv ? row : 0)) * K + (size_t)it.kc * d.Kc + chunk * 16;
                for (int s0 = 0; s0 < nks; s0 += 8) {
                    uint4 v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        v[u] = (rv && s0 + u < nks) ? ldg128(src + (s0 + u) * 128) : make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (s0 + u < nks)
                            *reinterpret_cast<uint4 *>(Bsm + (s0 + u) * BSTEP + sw128_offset(row, chunk)) = v[u];
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                const bool tv = lane < it.ntok;
                for (int g = 0; g < nks; ++g) {
                    uint32_t w = 0x7f7f7f7fu;
                    if (tv) w = 0x01010101u * d.a_s[(size_t)(it.tok0 + lane) * kb_all + it.kc * nks + g];
                    tmem_st4(tm + lane_base + COL_SFB + 4 * g, w, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
                }
                tmem_wait_st();
                fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(B.b_ready);
                ++nb;
                key = it.key;
            }
            // weight scale factors of this item
            if (q >= 2 && !twait(B.sfa_free + buf, ((q >> 1) - 1) & 1, d.err, B.abort)) break;
            fence_after_sync();
            for (int g0 = 0; g0 < nks; g0 += 8) {
                uint32_t w[8][4];
#pragma unroll
                for (int gg = 0; gg < 8; ++gg) {
                    const int g = g0 + gg;
#pragma unroll
                    for (int r1 = 0; r1 < 4; ++r1) {
                        const int r = it.tile * 128 + 32 * r1 + lane;
                        uint32_t x = 0x7f7f7f7fu;
                        if (g < nks) {
                            if (d.fp4) {
                                x = __ldg(reinterpret_cast<const uint32_t *>(d.w_s + (size_t)r * (K / 32) +
                                                                             (size_t)it.kc * (d.Kc / 32)) + g);
                            } else {
                                x = 0x01010101u * d.w_s[(size_t)(r / 128) * kb_all + it.kc * nks + g];
                            }
                        }
                        w[gg][r1] = x;
                    }
                }
#pragma unroll
                for (int gg = 0; gg < 8; ++gg)
                    if (g0 + gg < nks)
                        tmem_st4(tm + lane_base + COL_SFA + 128 * buf + 4 * (g0 + gg), w[gg][0], w[gg][1],
                                 w[gg][2], w[gg][3]);
            }
            tmem_wait_st();
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(B.sfa_ready + buf);
            if (qprev >= 0) epilogue(qprev, prev);
            prev = it;
            qprev = q;
        }
        if (qprev >= 0 && !*B.abort) epilogue(qprev, prev);
    }
    fence_before_sync();
    __syncthreads();
    if (warp == W_MMA) {
        fence_after_sync();
        tmem_dealloc(tm, 512);
    }
}

// ---------------------------------------------------------------------------
// The same GEMM with float32 block scales (fp8_gemm with scale_dtype float32,
// torch_ops.py:93-99): the tensor cores cannot apply a non-power-of-two scale, so
// each 128-wide K step's product goes into a fresh TMEM accumulator (unit UE8M0
// scales) and the worker warps add sa[m, kb] * sw[n / 128, kb] * D_step to fp32
// registers, in K order.  E4M3 weights only; ring of NACC step accumulators.
// ---------------------------------------------------------------------------
constexpr int NACC = 8;                      // step accumulators in flight
constexpr uint32_t COL_ACC = 0;              // NACC x 16 columns
constexpr uint32_t COL_UNIT = 128;           // unit scale factors (4 columns)
constexpr int F32_NBAR = 2 * STAGES + 2 + 2 * NACC + 1;  // ..., fin
constexpr int F32_OFF_SA = OFF_BAR + F32_NBAR * 8 + 64;  // [NTOK][KC_MAX / 128] f32 activation scales
constexpr int F32_SMEM = F32_OFF_SA + NTOK * (KC_MAX / 128) * 4 + 1024;
static_assert(F32_SMEM <= 232448, "shared memory budget");

struct DenseF32Args {
    CUtensorMap tmA;     // weights e4m3 [N, K], box 128 x 128, 128-byte swizzle
    const uint8_t *a;    // e4m3 tokens [M, K]
    const float *a_s;    // [M, K/128]
    const float *w_s;    // [ceil(N/128), K/128]
    int M, N, K, nkc, Kc;
    __nv_bfloat16 *out;  // [M, N]
    float *part;         // [nkc, M, N] (nkc > 1)
    unsigned *cnt;       // (nkc > 1)
    int *err;
};

__global__ void __launch_bounds__(THREADS, 1) k_dense_tc_f32(const __grid_constant__ DenseF32Args d) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bar = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    uint64_t *full = bar, *empty = bar + STAGES, *b_ready = bar + 2 * STAGES, *b_free = bar + 2 * STAGES + 1;
    uint64_t *acc_ready = bar + 2 * STAGES + 2, *acc_free = bar + 2 * STAGES + 2 + NACC;
    uint64_t *fin = bar + 2 * STAGES + 2 + 2 * NACC;
    uint32_t *tmem_base = reinterpret_cast<uint32_t *>(bar + F32_NBAR);
    volatile int *abort = reinterpret_cast<volatile int *>(bar + F32_NBAR) + 1;
    float *sa_s = reinterpret_cast<float *>(base + F32_OFF_SA);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        mbar_init(b_ready, 4);
        mbar_init(b_free, 1);
        for (int j = 0; j < NACC; ++j) { mbar_init(acc_ready + j, 1); mbar_init(acc_free + j, 4); }
        mbar_init(fin, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) { tmem_alloc(tmem_base, 256); tmem_relinquish(); }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = *tmem_base;
    const int ntile = d.N / 128, ntg = (d.M + NTOK - 1) / NTOK;
    const int n = d.nkc * ntg * ntile;
    const int i0 = (int)(((long long)n * blockIdx.x) / gridDim.x);
    const int i1 = (int)(((long long)n * (blockIdx.x + 1)) / gridDim.x);
    const int nks = d.Kc / 128;
    uint8_t *Bsm = base + OFF_B;
    DenseArgs geo;  // item decoding only
    geo.M = d.M; geo.N = d.N; geo.nkc = d.nkc;

    if (warp == W_PROD) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int gs = 0;
            for (int i = i0; i < i1 && !*abort; ++i) {
                const DItem it = dense_item(geo, i);
                for (int s = 0; s < nks; ++s, ++gs) {
                    const int st = gs % STAGES;
                    if (gs == STAGES) pdl_wait();
                    if (gs >= STAGES && !twait(empty + st, ((gs / STAGES) - 1) & 1, d.err, abort)) break;
                    mbar_arrive_expect_tx(full + st, ABOX);
                    tma_load_2d_hint(base + st * ABOX, &d.tmA, it.kc * d.Kc + s * 128, it.tile * 128, full + st,
                                     pol);
                }
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            pdl_wait();
            int gs = 0, nb = 0, key = -1;
            for (int i = i0; i < i1 && !*abort; ++i) {
                const DItem it = dense_item(geo, i);
                if (it.key != key) {
                    if (!twait(b_ready, nb & 1, d.err, abort)) break;
                    ++nb;
                    key = it.key;
                }
                bool ok = true;
                for (int s = 0; s < nks; ++s, ++gs) {
                    const int st = gs % STAGES, ab = gs % NACC;
                    if (gs >= NACC && !twait(acc_free + ab, ((gs / NACC) - 1) & 1, d.err, abort)) { ok = false; break; }
                    if (!twait(full + st, (gs / STAGES) & 1, d.err, abort)) { ok = false; break; }
                    fence_after_sync();
                    const uint64_t ad = smem_desc_sw128(base + st * ABOX);
                    const uint64_t bd = smem_desc_sw128(Bsm + s * BSTEP);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        mma_mxf8f6f4(tm + COL_ACC + 16 * ab, ad + 2 * j, bd + 2 * j, idesc_mxf8f6f4(0, 0, NTOK, j),
                                     tm + COL_UNIT, tm + COL_UNIT, j != 0);
                    commit(empty + st);
                    commit(acc_ready + ab);
                }
                if (!ok) break;
                const bool last_of_set = (i + 1 >= i1) || dense_item(geo, i + 1).key != it.key;
                if (last_of_set) commit(b_free);
            }
            // all of this thread's MMAs complete before TMEM is released
            commit(fin);
            wf_wait(fin, 0, d.err);
        }
    } else {
        pdl_wait();
        const int wq = warp & 3;
        const int wt = threadIdx.x - W_WORK0 * 32;
        const uint32_t lane_base = (uint32_t)(32 * wq) << 16;
        const int K = d.K, kb_all = K / 128;
        // unit scale factors (2^0) for both operands, every lane
        tmem_st4(tm + lane_base + COL_UNIT, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
        tmem_wait_st();
        fence_before_sync();
        int nb = 0, key = -1, gs = 0;
        bool dead = false;
        for (int i = i0; i < i1 && !dead; ++i) {
            if (*abort) break;
            const DItem it = dense_item(geo, i);
            if (it.key != key) {
                if (nb > 0 && !twait(b_free, (nb - 1) & 1, d.err, abort)) break;
                const int row = wt >> 3, chunk = wt & 7;
                const bool rv = row < it.ntok;
                const uint8_t *src = d.a + (size_t)(it.tok0 + (rv ? row : 0)) * K + (size_t)it.kc * d.Kc + chunk * 16;
                for (int s0 = 0; s0 < nks; s0 += 8) {
                    uint4 v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        v[u] = (rv && s0 + u < nks) ? ldg128(src + (s0 + u) * 128) : make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (s0 + u < nks)
                            *reinterpret_cast<uint4 *>(Bsm + (s0 + u) * BSTEP + sw128_offset(row, chunk)) = v[u];
                }
                // the token group's activation scales of this K chunk
                bar_sync(1, 128);  // the previous group's epilogue read sa_s
                for (int k = wt; k < NTOK * nks; k += 128) {
                    const int m = k / nks, s = k - m * nks;
                    sa_s[k] = m < it.ntok ? __ldg(d.a_s + (size_t)(it.tok0 + m) * kb_all + it.kc * nks + s) : 0.f;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                bar_sync(1, 128);
                fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(b_ready);
                ++nb;
                key = it.key;
            }
            const int row = it.tile * 128 + 32 * wq + lane;
            float acc[NTOK];
#pragma unroll
            for (int m = 0; m < NTOK; ++m) acc[m] = 0.f;
            for (int s = 0; s < nks; ++s, ++gs) {
                const int ab = gs % NACC;
                const float sw = __ldg(d.w_s + (size_t)(row / 128) * kb_all + it.kc * nks + s);
                if (!twait(acc_ready + ab, (gs / NACC) & 1, d.err, abort)) { dead = true; break; }
                fence_after_sync();
                uint32_t v[16];
                tmem_ld16(tm + lane_base + COL_ACC + 16 * ab, v);
                tmem_wait_ld();
                fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_free + ab);
#pragma unroll
                for (int m = 0; m < NTOK; ++m) acc[m] += (sa_s[m * nks + s] * sw) * __uint_as_float(v[m]);
            }
            if (dead) break;
            if (d.nkc == 1) {
#pragma unroll
                for (int m = 0; m < NTOK; ++m)
                    if (m < it.ntok) d.out[(size_t)(it.tok0 + m) * d.N + row] = __float2bfloat16_rn(acc[m]);
            } else {
#pragma unroll
                for (int m = 0; m < NTOK; ++m)
                    if (m < it.ntok) d.part[((size_t)it.kc * d.M + it.tok0 + m) * d.N + row] = acc[m];
                __threadfence();
                __syncwarp();
                unsigned *cnt = d.cnt + ((size_t)it.tg * ntile + it.tile) * 4 + wq;
                int last = 0;
                if (lane == 0) last = atomicAdd(cnt, 1u) == (unsigned)d.nkc - 1;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    float sum[NTOK];
#pragma unroll
                    for (int m = 0; m < NTOK; ++m) sum[m] = 0.f;
                    for (int c = 0; c < d.nkc; ++c) {
                        const float *pc = d.part + ((size_t)c * d.M + it.tok0) * d.N + row;
#pragma unroll
                        for (int m = 0; m < NTOK; ++m) sum[m] += m < it.ntok ? __ldcg(pc + (size_t)m * d.N) : 0.f;
                    }
#pragma unroll
                    for (int m = 0; m < NTOK; ++m)
                        if (m < it.ntok) d.out[(size_t)(it.tok0 + m) * d.N + row] = __float2bfloat16_rn(sum[m]);
                    if (lane == 0) *cnt = 0u;
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == W_MMA) {
        fence_after_sync();
        tmem_dealloc(tm, 256);
    }
}

}  // namespace tc
}  // namespace wf
