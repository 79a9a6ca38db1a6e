// wf_moe.cu - B200 (sm_100a) kernels of the WANferenz MoE decode layer and
// the C ABI declared in include/wfb200.h.
//
// The layer (wanferenz/model/architecture.py:674-794) runs as three
// persistent launches of one CTA per SM:
//
//   K1 "up"   router logits (fp64 accumulation) + top-k/dispatch tables by the
//             last router CTA; shared-expert w1/w3 + SwiGLU  -> hs (bf16)
//   K2 "mid"  routed-expert w1/w3 + SwiGLU * route weight     -> h  (bf16)
//             shared-expert w2                                  -> os (bf16)
//   K3 "down" routed-expert w2                                  -> o  (bf16)
//             + per-row-block ascending-expert combine          -> y
//
// Each launch is a static, balanced split of "items" over the CTAs.  An item
// is up to 32 weight rows (<= 34 KB) times up to 16 tokens.  Inside a CTA one
// producer warp streams each item's rows into a 5-slot shared-memory ring with
// bulk TMA copies (cp.async.bulk, completion on an mbarrier); eight consumer
// warps split K, dequantize FP4 in registers with integer ops (E2M1 -> E4M3
// of value x 2^-6, exact; FP8 weights need no conversion), multiply on the
// tensor cores (mma.m16n8k32 E4M3 x E4M3 -> f32), apply the per-32 weight and
// per-128 activation scales in f32, and reduce across warps in a fixed order
// through shared memory.
// Activations are quantized to E4M3 (act_quant, torch_ops.py:33-49) by the
// consumer warps themselves when they load a token's K-slice.

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../../include/wfb200.h"
#include "wf_ptx.cuh"
#include "wf_tc.cuh"

namespace wf {

constexpr int NCW = 8;                 // consumer warps
constexpr int NTHR = (NCW + 1) * 32;   // + 1 producer warp
constexpr int NCT = NCW * 32;          // consumer threads
constexpr int NSLOT = 5;               // ring slots
constexpr int SLOT_W = 34816;          // weight bytes per slot (padded rows)
constexpr int SLOT_S = 2048;           // FP4 scale bytes per slot
constexpr int SLOT_BYTES = SLOT_W + SLOT_S;
constexpr int MAXR = 32;               // weight rows per item
constexpr int NTM = 2;                 // n-tiles (8 tokens each) per item
constexpr int TPI = 8 * NTM;           // tokens per item
constexpr int SPW = 4;                 // max 128-wide K segments per warp
constexpr int KMAX = NCW * SPW * 128;  // longest K one item covers (4096)
constexpr int RED_BYTES = NCW * MAXR * TPI * 4;
constexpr int OFF_RED = NSLOT * SLOT_BYTES;
constexpr int OFF_BAR = OFF_RED + RED_BYTES;
constexpr int OFF_MISC = OFF_BAR + 2 * NSLOT * 8 + 64;
constexpr int MISC_BYTES = 2048;  // router partial sums (fp64) / top-k expert counts
constexpr int MAX_E = 512;
constexpr int MAX_K = 8;
constexpr int MAX_T = 256;
constexpr int MAX_PAIRS = MAX_T * MAX_K;
// routing tables copied to shared memory at kernel start (K2, K3)
constexpr int OFF_ROUTE = OFF_MISC + MISC_BYTES;
constexpr int ROUTE_TABLE_BYTES = 3 * (MAX_E + 1) * 4 + MAX_PAIRS * 2 + MAX_PAIRS * 4;
// the router CTA's top-k uses the same region: token bitmaps, pair offsets, scan scratch
constexpr int TOPK_ROUTE_BYTES = MAX_E * (MAX_T / 32) * 4 + MAX_E * 4 + NCW * 8;
constexpr int ROUTE_BYTES = ROUTE_TABLE_BYTES > TOPK_ROUTE_BYTES ? ROUTE_TABLE_BYTES : TOPK_ROUTE_BYTES;
constexpr int SMEM_BYTES = OFF_ROUTE + ROUTE_BYTES;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

constexpr int EP_MAX_RANKS = 8;  // expert-parallel ranks over peer memory
constexpr int EP_CTR = 2 * EP_MAX_RANKS;       // flag word: epoch of the last completed forward
constexpr int EP_FIN = 2 * EP_MAX_RANKS + 1;   // flag word: finish blocks done
constexpr int EP_FLAG_WORDS = 2 * EP_MAX_RANKS + 2;

enum { EP_RSWIGLU = 1, EP_SSWIGLU = 2, EP_SOUT = 3, EP_ROUT = 4, EP_DENSE = 5 };
enum { BS_XPAIR = 1, BS_XTOK = 2, BS_H = 3, BS_HS = 4, BS_PREQ = 5 };
enum { FMT_FP4 = 0, FMT_FP8 = 1 };
enum { KID_UP = 1, KID_MID = 2, KID_DOWN = 3, KID_DENSE = 4 };

// hdr fields written by the top-k CTA
enum { H_NACT = 0, H_IT2 = 1, H_IT3 = 2, H_TGT = 3, H_NPAIR = 4, H_SIZE = 8 };

struct Geo {
    int st_w13, st_w2, st_s13, st_s2;  // smem row strides (bytes)
    int nh13, r2, nhs13, rs2;          // rows per item
};

struct MoeArgs {
    int T, D, I, E, El, e0, topk, score_func, hash, ue8m0, partial, shared_f32, route_only;
    float route_scale, swiglu_limit;
    long long vocab;
    const __nv_bfloat16 *x;
    const long long *ids;
    const __nv_bfloat16 *gate_w;
    const float *gate_b;
    const int *tid2eid;
    const uint8_t *w13, *w13_s, *w2, *w2_s, *sw13, *sw2;
    const void *ss13, *ss2;
    __nv_bfloat16 *y;
    float *y_partial;
    float *out_w;
    long long *out_idx;
    // workspace
    float *logits;
    int *hdr, *act_expert, *act_off, *act_it2, *act_it3;
    int *pair_tok, *tok_np, *tok_pairs, *ridx;
    float *pair_w, *rw;
    __nv_bfloat16 *h, *hs, *o, *os;
    unsigned *cnt_router, *cnt_rb;
    int *err;
    Geo g;
    int tc;              // expert phases on tcgen05 (k_moe_tc): K1 quantizes x, skips the shared expert
    uint8_t *xq, *xs;    // E4M3 tokens [T, D] and their e8m0 scales [T, D/128] (tc)
    // routing given by the caller (wf_moe_forward_ep): no router, in_w / in_idx instead
    int given;
    const float *in_w;         // [T, topk] routing weights
    const long long *in_idx;   // [T, topk] global expert ids
    // the shared expert runs on rows [sh0, sh0 + shT); sh_add: the combine adds those
    // rows to the output (whole layer: all rows; partial forward: none, wf_moe_finish
    // adds them; expert-parallel: the rank's own rows of the gathered batch)
    int sh0, shT, sh_add;
    // bound (SM cycles) of waits on another role's progress (wf_set_wait_limit)
    long long wait_limit;
    // expert parallelism over peer memory (wf_moe_forward_ep_p2p, fused engine only):
    // this rank routes its own Tr tokens, which are rows [ep_rank * Tr, +Tr) of the
    // gathered batch of T = ep_world * Tr rows; the buffers below are every rank's
    // (index ep_rank is this rank's own, in local memory)
    int ep, ep_rank, ep_world, Tr;
    uint8_t *ep_xq[EP_MAX_RANKS];     // gathered E4M3 tokens [T, D]
    uint8_t *ep_xs[EP_MAX_RANKS];     // their e8m0 scales [T, D/128]
    int *ep_ridx[EP_MAX_RANKS];       // gathered routing [T, topk] expert ids
    float *ep_rw[EP_MAX_RANKS];       // and weights
    float *ep_yrecv[EP_MAX_RANKS];    // partial rows of the owner's tokens from every rank [P][Tr][D]
    // [0, P): dispatch epochs, [EP_MAX_RANKS, +P): combine epochs, [EP_CTR]: the
    // epoch of the last completed forward (this rank's; read at the start)
    unsigned *ep_flags[EP_MAX_RANKS];
    unsigned *ep_done;                // local: 256-row output blocks combined in this launch
};

// Dense GEMM (operator entry points) arguments.
struct DenseArgs {
    int M, N, K, G;               // G > 0: grouped (slot g uses weights g, token g)
    int wfmt, a_f32, b_f32;       // weight format; scale kinds
    const uint8_t *a;             // e4m3 [M, K]
    const void *a_s;              // [M, K/128]
    const uint8_t *b;             // weights
    const void *b_s;              // scales
    __nv_bfloat16 *out;           // [M, N]
    int rows, stride;             // rows per item, smem row stride
    int nkc, Kc;                  // K chunks (split-K) and chunk length
    float *part;                  // [nkc, M, N] fp32 partials (nkc > 1)
    unsigned *cnt;                // [M-groups * N/rows] arrival counters (nkc > 1)
    int *err;
};

struct Item {
    int ep, bsrc, fmt, K, stride;  // K: columns this item covers
    int nrun, rrows;
    int gpitch, spitch;            // global bytes between consecutive weight / scale rows
    int kb0, kc;                   // first 128-block of K this item covers, K chunk index
    const uint8_t *wsrc[2];
    const uint8_t *ssrc[2];
    int grow[2];
    int row0, a, tok0, ntok, rb;
};

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// item decoding (identical in producer and consumers)
// ---------------------------------------------------------------------------
__device__ __forceinline__ Item decode_moe(int kid, const MoeArgs &a, int i, int ai, int n_it2,
                                           const int *act_expert, const int *act_off,
                                           const int *act_it) {
    Item it;
    const int D = a.D, I = a.I;
    it.ssrc[0] = it.ssrc[1] = nullptr;
    it.grow[0] = it.grow[1] = 0;
    it.rb = 0; it.kb0 = 0; it.kc = 0;
    if (kid == KID_UP) {  // shared expert w1/w3 rows + SwiGLU
        // token group outer, row block inner: a CTA's contiguous range keeps
        // one token group (its B fragments stay in registers)
        const int nh = a.g.nhs13, nhb = I / nh;
        const int tg = i / nhb, hb = i % nhb;
        it.ep = EP_SSWIGLU; it.bsrc = BS_XTOK; it.fmt = FMT_FP8; it.K = D; it.stride = a.g.st_s13;
        it.nrun = 2; it.rrows = nh; it.gpitch = D; it.spitch = 0;
        it.grow[0] = hb * nh; it.grow[1] = I + hb * nh;
        it.wsrc[0] = a.sw13 + (size_t)it.grow[0] * D;
        it.wsrc[1] = a.sw13 + (size_t)it.grow[1] * D;
        it.row0 = hb * nh; it.a = 0; it.tok0 = a.sh0 + tg * TPI; it.ntok = min(TPI, a.shT - tg * TPI);
        return it;
    }
    if (kid == KID_MID && i >= n_it2) {  // shared expert w2
        const int j = i - n_it2, nr = a.g.rs2, nrb = D / nr;
        const int tg = j / nrb, rb = j % nrb;
        it.ep = EP_SOUT; it.bsrc = BS_HS; it.fmt = FMT_FP8; it.K = I; it.stride = a.g.st_s2;
        it.nrun = 1; it.rrows = nr; it.gpitch = I; it.spitch = 0;
        it.grow[0] = rb * nr;
        it.wsrc[0] = a.sw2 + (size_t)it.grow[0] * I;
        it.wsrc[1] = it.wsrc[0];
        it.row0 = rb * nr; it.a = 0; it.tok0 = a.sh0 + tg * TPI; it.ntok = min(TPI, a.shT - tg * TPI);
        return it;
    }
    // routed items (tables in shared memory)
    const int local = i - act_it[ai];
    const int p0 = act_off[ai], ta = act_off[ai + 1] - p0;
    const int nblk = (kid == KID_MID) ? I / a.g.nh13 : D / a.g.r2;
    const int tg = local / nblk, blk = local % nblk;
    const int el = act_expert[ai] - a.e0;
    it.a = ai; it.tok0 = p0 + tg * TPI; it.ntok = min(TPI, ta - tg * TPI);
    if (kid == KID_MID) {  // routed w1/w3 rows + SwiGLU
        const int nh = a.g.nh13;
        const uint8_t *wb = a.w13 + (size_t)el * (2 * I) * (D / 2);
        const uint8_t *sb = a.w13_s + (size_t)el * (2 * I) * (D / 32);
        it.ep = EP_RSWIGLU; it.bsrc = BS_XPAIR; it.fmt = FMT_FP4; it.K = D; it.stride = a.g.st_w13;
        it.nrun = 2; it.rrows = nh; it.gpitch = D / 2; it.spitch = D / 32;
        it.grow[0] = blk * nh; it.grow[1] = I + blk * nh;
        it.wsrc[0] = wb + (size_t)it.grow[0] * (D / 2);
        it.wsrc[1] = wb + (size_t)it.grow[1] * (D / 2);
        it.ssrc[0] = sb + (size_t)it.grow[0] * (D / 32);
        it.ssrc[1] = sb + (size_t)it.grow[1] * (D / 32);
        it.row0 = blk * nh;
    } else {  // routed w2 rows
        const int nr = a.g.r2;
        const uint8_t *wb = a.w2 + (size_t)el * D * (I / 2);
        const uint8_t *sb = a.w2_s + (size_t)el * D * (I / 32);
        it.ep = EP_ROUT; it.bsrc = BS_H; it.fmt = FMT_FP4; it.K = I; it.stride = a.g.st_w2;
        it.nrun = 1; it.rrows = nr; it.gpitch = I / 2; it.spitch = I / 32;
        it.grow[0] = blk * nr;
        it.wsrc[0] = wb + (size_t)it.grow[0] * (I / 2);
        it.wsrc[1] = it.wsrc[0];
        it.ssrc[0] = sb + (size_t)it.grow[0] * (I / 32);
        it.ssrc[1] = it.ssrc[0];
        it.row0 = blk * nr; it.rb = blk;
    }
    return it;
}

__device__ __forceinline__ Item decode_dense(const DenseArgs &d, int i) {
    // order: K chunk, then token group (or group g), then row block fastest, so a
    // CTA's contiguous item range shares one activation slice (B in registers)
    Item it;
    const int nrb = d.N / d.rows;
    const int ntg = d.G > 0 ? d.G : cdiv(d.M, TPI);
    const int kc = i / (ntg * nrb), rem = i % (ntg * nrb);
    const int tg = rem / nrb, rb = rem % nrb;
    int tok0, ntok, gsel = 0;
    if (d.G > 0) { gsel = tg; tok0 = tg; ntok = 1; }
    else { tok0 = tg * TPI; ntok = min(TPI, d.M - tok0); }
    it.ep = EP_DENSE; it.bsrc = BS_PREQ; it.fmt = d.wfmt; it.K = d.Kc; it.stride = d.stride;
    it.nrun = 1; it.rrows = d.rows; it.rb = tg * nrb + rb; it.kc = kc;
    it.kb0 = kc * (d.Kc / 128);
    it.grow[0] = rb * d.rows; it.grow[1] = 0;
    const size_t rowb = d.wfmt == FMT_FP4 ? (size_t)d.K / 2 : (size_t)d.K;
    it.gpitch = (int)rowb;
    const uint8_t *wbase = d.b + (size_t)gsel * d.N * rowb;
    const size_t koff = d.wfmt == FMT_FP4 ? (size_t)kc * d.Kc / 2 : (size_t)kc * d.Kc;
    it.wsrc[0] = wbase + (size_t)it.grow[0] * rowb + koff;
    it.wsrc[1] = it.wsrc[0];
    if (d.wfmt == FMT_FP4) {
        it.spitch = d.K / 32;
        const uint8_t *sbase = (const uint8_t *)d.b_s + (size_t)gsel * d.N * (d.K / 32);
        it.ssrc[0] = sbase + (size_t)it.grow[0] * (d.K / 32) + (size_t)kc * d.Kc / 32;
    } else {
        it.spitch = 0;
        it.ssrc[0] = nullptr;
    }
    it.ssrc[1] = it.ssrc[0];
    it.row0 = it.grow[0]; it.a = gsel * 65536 + kc; it.tok0 = tok0; it.ntok = ntok;
    return it;
}

// ---------------------------------------------------------------------------
// shared-memory context
// ---------------------------------------------------------------------------
struct Smem {
    uint8_t *base;
    __device__ uint8_t *slot(int s) const { return base + s * SLOT_BYTES; }
    __device__ float *red() const { return reinterpret_cast<float *>(base + OFF_RED); }
    __device__ uint64_t *full(int s) const { return reinterpret_cast<uint64_t *>(base + OFF_BAR) + s; }
    __device__ uint64_t *empty(int s) const {
        return reinterpret_cast<uint64_t *>(base + OFF_BAR) + NSLOT + s;
    }
    __device__ volatile int *flags() const {
        return reinterpret_cast<volatile int *>(base + OFF_BAR + 2 * NSLOT * 8);
    }
    __device__ double *misc() const { return reinterpret_cast<double *>(base + OFF_MISC); }
};

// Routing tables of the current forward, in shared memory.
struct RouteSm {
    int *act_expert, *act_off, *act_it;
    int16_t *pair_tok;
    float *pair_w;
};

__device__ __forceinline__ RouteSm route_sm(const Smem &sm) {
    RouteSm r;
    int *b = reinterpret_cast<int *>(sm.base + OFF_ROUTE);
    r.act_expert = b;
    r.act_off = b + (MAX_E + 1);
    r.act_it = b + 2 * (MAX_E + 1);
    r.pair_tok = reinterpret_cast<int16_t *>(b + 3 * (MAX_E + 1));
    r.pair_w = reinterpret_cast<float *>(r.pair_tok + MAX_PAIRS);
    return r;
}

// All 288 threads: copy the tables written by the router CTA (K1) into shared memory.
__device__ __forceinline__ void load_route(const Smem &sm, const int *act_expert, const int *act_off,
                                           const int *act_it, const int *pair_tok, const float *pair_w,
                                           int n_act, int n_pairs) {
    const RouteSm r = route_sm(sm);
    for (int i = threadIdx.x; i <= n_act; i += blockDim.x) {
        r.act_off[i] = act_off[i];
        r.act_it[i] = act_it[i];
        if (i < n_act) r.act_expert[i] = act_expert[i];
    }
    for (int i = threadIdx.x; i < n_pairs; i += blockDim.x) {
        r.pair_tok[i] = (int16_t)pair_tok[i];
        r.pair_w[i] = pair_w[i];
    }
    __syncthreads();
}

// Walks a CTA's contiguous item range; `ai` tracks the active expert of item `i`.
struct Cursor {
    int i, ai;
};

__device__ __forceinline__ Cursor cursor_at(const RouteSm &r, int n_act, int i) {
    int lo = 0, hi = n_act - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (r.act_it[mid] <= i) lo = mid; else hi = mid - 1;
    }
    return Cursor{i, lo};
}

__device__ __forceinline__ void cursor_next(const RouteSm &r, int n_act, Cursor &c) {
    ++c.i;
    while (c.ai + 1 < n_act && c.i >= r.act_it[c.ai + 1]) ++c.ai;
}

__device__ __forceinline__ void item_range(int n, int &i0, int &i1) {
    i0 = (int)(((long long)n * blockIdx.x) / gridDim.x);
    i1 = (int)(((long long)n * (blockIdx.x + 1)) / gridDim.x);
}

// ---------------------------------------------------------------------------
// producer: stream each item's weight rows (and FP4 scales) into the ring
// ---------------------------------------------------------------------------
template <typename Decode>
__device__ void produce(const Smem &sm, int i0, int i1, int *err, long long lim, Decode decode) {
    if ((threadIdx.x & 31) != 0) return;
    volatile int *abort = sm.flags();
    int q = 0, armed = 0;  // items walked; items whose copies were issued (a prefix)
    for (int i = i0; i < i1; ++i, ++q) {
        const Item it = decode(i);
        const int s = q % NSLOT;
        if (q >= NSLOT && !*abort) {
            if (!wf_wait(sm.empty(s), ((q / NSLOT) - 1) & 1, err, lim)) *abort = 1;
        }
        if (*abort) continue;
        ++armed;
        const uint32_t rowb = it.fmt == FMT_FP4 ? it.K / 2 : it.K;
        const uint32_t ks = it.K / 32;
        const int na = it.nrun * it.rrows;
        uint32_t bytes = na * rowb + (it.fmt == FMT_FP4 ? na * ks : 0);
        mbar_arrive_expect_tx(sm.full(s), bytes);
        uint8_t *dst = sm.slot(s);
#pragma unroll
        for (int run = 0; run < 2; ++run) {
            if (run >= it.nrun) break;
            const uint8_t *wsrc = run ? it.wsrc[1] : it.wsrc[0];
            const uint8_t *ssrc = run ? it.ssrc[1] : it.ssrc[0];
            for (int r = 0; r < it.rrows; ++r)
                bulk_g2s(dst + (run * it.rrows + r) * it.stride, wsrc + (size_t)r * it.gpitch, rowb,
                         sm.full(s));
            if (it.fmt == FMT_FP4) {
                if ((uint32_t)it.spitch == ks) {  // the run's scale rows are contiguous
                    bulk_g2s(dst + SLOT_W + run * it.rrows * ks, ssrc, it.rrows * ks, sm.full(s));
                } else {  // split-K chunk: one copy per row (ks is a multiple of 16 here)
                    for (int r = 0; r < it.rrows; ++r)
                        bulk_g2s(dst + SLOT_W + (run * it.rrows + r) * ks,
                                 ssrc + (size_t)r * it.spitch, ks, sm.full(s));
                }
            }
        }
    }
    // drain: every armed phase must complete before the CTA may exit (after an
    // abort only the first `armed` items were issued)
    const int nq = armed;
    for (int s = 0; s < NSLOT && s < nq; ++s) {
        const int last = s + ((nq - 1 - s) / NSLOT) * NSLOT;
        wf_wait(sm.full(s), (last / NSLOT) & 1, err);
    }
}

// ---------------------------------------------------------------------------
// consumers
// ---------------------------------------------------------------------------
struct BRegs {
    // token slot g's K-slice as packed E4M3 codes: per 128-wide segment, per
    // 32-block j, the two m16n8k32 B registers {b0, b1} (see arrange_codes)
    uint32_t b[NTM][SPW][8];
    float sx[NTM][SPW][2];  // activation scales of the C-fragment tokens (x 2^6 for FP4 items)
};

__device__ __forceinline__ float round_scale_e8(float amax, int ue8m0) {
    const float x = amax * (1.0f / 448.0f);
    if (!ue8m0) return x;
    const uint32_t b = __float_as_uint(x);
    if ((b & 0x7fffffu) == 0) return x;
    return __uint_as_float(((b >> 23) + 1) << 23);
}

// 8 E4M3 codes (lo = elements 0-3, hi = 4-7) -> the thread's two B registers.
// FP4 items pair the MMA k-slots with even / odd elements (the even-odd split
// of fp4_to_e4m3); FP8 items with the two contiguous halves.
__device__ __forceinline__ void arrange_codes(uint32_t lo, uint32_t hi, bool interleave,
                                              uint32_t &b0, uint32_t &b1) {
    if (interleave) {
        b0 = __byte_perm(lo, hi, 0x6420);  // elements 0, 2, 4, 6
        b1 = __byte_perm(lo, hi, 0x7531);  // elements 1, 3, 5, 7
    } else {
        b0 = lo;
        b1 = hi;
    }
}

// act_quant (torch_ops.py:33-49) of one token's 128-block, held as 4 chunks of
// 8 bf16 per lane (chunk j = elements 32j + 8*tig .. +7); the quad's 4 lanes
// share the block amax.  Writes the 8 B registers; returns the block scale.
__device__ __forceinline__ float quant_seg(const __nv_bfloat16 *seg, int tig, bool valid, int ue8m0,
                                           bool interleave, uint32_t (&out)[8]) {
    uint4 w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        w[j] = valid ? ldg128(seg + 32 * j + 8 * tig) : make_uint4(0, 0, 0, 0);
    uint32_t amax_bits = 0;  // |bf16| max on bit patterns (sign cleared: order-preserving)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t v[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            amax_bits = max(amax_bits, v[e] & 0x7fffu);
            amax_bits = max(amax_bits, (v[e] >> 16) & 0x7fffu);
        }
    }
    float amax = bf16_bits_to_f32(amax_bits);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float s = round_scale_e8(fmaxf(amax, 1e-4f), ue8m0);
    const float inv = 1.0f / s;  // exact when s is a power of two
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t v[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
        uint32_t q[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float lo = bf16_bits_to_f32(v[e] & 0xffffu), hi = bf16_bits_to_f32(v[e] >> 16);
            if (ue8m0) { lo *= inv; hi *= inv; }
            else { lo = __fdiv_rn(lo, s); hi = __fdiv_rn(hi, s); }
            lo = fminf(fmaxf(lo, -448.f), 448.f);
            hi = fminf(fmaxf(hi, -448.f), 448.f);
            q[e] = f32x2_to_e4m3x2(lo, hi);  // 16 bits: element 2e low, 2e+1 high
        }
        const uint32_t lo4 = q[0] | (q[1] << 16), hi4 = q[2] | (q[3] << 16);
        arrange_codes(lo4, hi4, interleave, out[2 * j], out[2 * j + 1]);
    }
    return valid ? s : 0.f;
}

// Pre-quantized E4M3 codes of one 128-block (4 chunks of 8 bytes per lane).
__device__ __forceinline__ void codes_seg(const uint8_t *seg, int tig, bool valid, bool interleave,
                                          uint32_t (&out)[8]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint2 u = make_uint2(0, 0);
        if (valid) u = __ldg(reinterpret_cast<const uint2 *>(seg + 32 * j + 8 * tig));
        arrange_codes(u.x, u.y, interleave, out[2 * j], out[2 * j + 1]);
    }
}

template <typename RowPtr, typename PreqScale>
__device__ __forceinline__ void load_b(const Item &it, int warp, int lane, int ue8m0, BRegs &B,
                                       RowPtr rowptr, PreqScale preq_scale) {
    const int g = lane >> 2, tig = lane & 3;
    const int nseg = it.K / 128, spw = cdiv(nseg, NCW), s0 = warp * spw;
    const int nnt = cdiv(it.ntok, 8);
    const bool il = it.fmt == FMT_FP4;
    const float fold = il ? 64.f : 1.f;  // FP4 weights enter the MMA as E2M1 x 2^-6
#pragma unroll
    for (int nt = 0; nt < NTM; ++nt) {
        const int j = nt * 8 + g;
        const bool tv = (nt < nnt) && (j < it.ntok);
#pragma unroll
        for (int sj = 0; sj < SPW; ++sj) {
            const int s = s0 + sj;
            const bool sv = (sj < spw) && (s < nseg) && (nt < nnt);
            float sc = 0.f;
            if (sv) {
                if (it.bsrc == BS_PREQ) {
                    const uint8_t *src = tv ? (const uint8_t *)rowptr(it, j) : nullptr;
                    codes_seg(src ? src + s * 128 : nullptr, tig, tv, il, B.b[nt][sj]);
                    sc = tv ? preq_scale(it, j, s) : 0.f;
                } else {
                    const __nv_bfloat16 *src = tv ? (const __nv_bfloat16 *)rowptr(it, j) : nullptr;
                    sc = quant_seg(tv ? src + s * 128 : nullptr, tig, tv, ue8m0, il, B.b[nt][sj]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) B.b[nt][sj][e] = 0u;
            }
            sc *= fold;
            B.sx[nt][sj][0] = __shfl_sync(0xffffffffu, sc, (2 * tig) * 4);
            B.sx[nt][sj][1] = __shfl_sync(0xffffffffu, sc, (2 * tig + 1) * 4);
        }
    }
}

// 8 packed E2M1 codes -> E4M3 bytes of value x 2^-6, split by element parity:
// even elements (low nibbles) into `ev`, odd (high nibbles) into `od`.  An
// E2M1 nibble s|e1 e0 m moved to bits s|.|.|.|e1 e0 m|.|. of a byte is the E4M3
// encoding of its value x 2^-6, subnormal 0.5 included, so this is exact.
__device__ __forceinline__ void fp4_to_e4m3(uint32_t w, uint32_t &ev, uint32_t &od) {
    const uint32_t a = w << 2;  // low-nibble magnitude -> bits 4..2, its sign -> bit 5
    ev = (a & 0x1c1c1c1cu) | ((a & 0x20202020u) << 2);
    const uint32_t c = w >> 2;  // high-nibble magnitude -> bits 4..2, its sign -> bit 5
    od = (c & 0x1c1c1c1cu) | ((c & 0x20202020u) << 2);
}

// FP8 block scale of global weight row `grow`, K-block `kb`
template <typename FP8Scale>
__device__ __forceinline__ float fp8_row_scale(const Item &it, int arow, int kb, FP8Scale f8s) {
    const int run = arow >= it.rrows;
    const int grow = (run ? it.grow[1] : it.grow[0]) + (arow - run * it.rrows);
    return f8s(grow / 128, it.kb0 + kb);
}

__device__ __forceinline__ void mma_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One item's main loop for one consumer warp: acc[m][nt][c] over the warp's K segments.
// Per 32-block j of segment s, lane (g, tig) supplies rows g and g+8, elements
// 8*tig .. 8*tig+7 of the block (one 32-bit word of FP4, 8 bytes of FP8).
template <typename FP8Scale>
__device__ __forceinline__ void compute_item(const Item &it, const uint8_t *slot, int warp,
                                             int lane, const BRegs &B, float (&acc)[2][NTM][4],
                                             FP8Scale f8s) {
    const int g = lane >> 2, tig = lane & 3;
    const int nseg = it.K / 128, spw = cdiv(nseg, NCW), s0 = warp * spw;
    const int na = it.nrun * it.rrows, nmt = cdiv(na, 16), nnt = cdiv(it.ntok, 8);
    const uint8_t *sc = slot + SLOT_W;
    const int ks = it.K / 32;
#pragma unroll
    for (int sj = 0; sj < SPW; ++sj) {
        const int s = s0 + sj;
        if (!(sj < spw && s < nseg)) continue;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            if (m >= nmt) continue;
            const int ra = 16 * m + g, rb = ra + 8;
            const bool va = ra < na, vb = rb < na;
            float cs[NTM][4];
#pragma unroll
            for (int nt = 0; nt < NTM; ++nt)
#pragma unroll
                for (int c = 0; c < 4; ++c) cs[nt][c] = 0.f;
            if (it.fmt == FMT_FP4) {
                // the 4 per-32 scales of this segment, one byte per block j
                const uint32_t sa4 = va ? *reinterpret_cast<const uint32_t *>(sc + ra * ks + s * 4) : 0u;
                const uint32_t sb4 = vb ? *reinterpret_cast<const uint32_t *>(sc + rb * ks + s * 4) : 0u;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int off = s * 64 + j * 16 + tig * 4;
                    const uint32_t wa = va ? *reinterpret_cast<const uint32_t *>(slot + ra * it.stride + off) : 0u;
                    const uint32_t wb = vb ? *reinterpret_cast<const uint32_t *>(slot + rb * it.stride + off) : 0u;
                    uint32_t a0, a2, a1, a3;
                    fp4_to_e4m3(wa, a0, a2);
                    fp4_to_e4m3(wb, a1, a3);
                    float d[NTM][4];
#pragma unroll
                    for (int nt = 0; nt < NTM; ++nt) {
#pragma unroll
                        for (int c = 0; c < 4; ++c) d[nt][c] = 0.f;
                        if (nt < nnt) mma_e4m3(d[nt], a0, a1, a2, a3, B.b[nt][sj][2 * j], B.b[nt][sj][2 * j + 1]);
                    }
                    const float fa = __uint_as_float(((sa4 >> (8 * j)) & 0xffu) << 23);
                    const float fb = __uint_as_float(((sb4 >> (8 * j)) & 0xffu) << 23);
#pragma unroll
                    for (int nt = 0; nt < NTM; ++nt) {
                        cs[nt][0] = fmaf(d[nt][0], fa, cs[nt][0]);
                        cs[nt][1] = fmaf(d[nt][1], fa, cs[nt][1]);
                        cs[nt][2] = fmaf(d[nt][2], fb, cs[nt][2]);
                        cs[nt][3] = fmaf(d[nt][3], fb, cs[nt][3]);
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NTM; ++nt) {
                    acc[m][nt][0] = fmaf(cs[nt][0], B.sx[nt][sj][0], acc[m][nt][0]);
                    acc[m][nt][1] = fmaf(cs[nt][1], B.sx[nt][sj][1], acc[m][nt][1]);
                    acc[m][nt][2] = fmaf(cs[nt][2], B.sx[nt][sj][0], acc[m][nt][2]);
                    acc[m][nt][3] = fmaf(cs[nt][3], B.sx[nt][sj][1], acc[m][nt][3]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int off = s * 128 + j * 32 + tig * 8;
                    uint2 wa = make_uint2(0, 0), wb = wa;
                    if (va) wa = *reinterpret_cast<const uint2 *>(slot + ra * it.stride + off);
                    if (vb) wb = *reinterpret_cast<const uint2 *>(slot + rb * it.stride + off);
#pragma unroll
                    for (int nt = 0; nt < NTM; ++nt)
                        if (nt < nnt) mma_e4m3(cs[nt], wa.x, wb.x, wa.y, wb.y, B.b[nt][sj][2 * j], B.b[nt][sj][2 * j + 1]);
                }
                const float fsa = va ? fp8_row_scale(it, ra, s, f8s) : 0.f;
                const float fsb = vb ? fp8_row_scale(it, rb, s, f8s) : 0.f;
#pragma unroll
                for (int nt = 0; nt < NTM; ++nt) {
                    acc[m][nt][0] = fmaf(cs[nt][0], fsa * B.sx[nt][sj][0], acc[m][nt][0]);
                    acc[m][nt][1] = fmaf(cs[nt][1], fsa * B.sx[nt][sj][1], acc[m][nt][1]);
                    acc[m][nt][2] = fmaf(cs[nt][2], fsb * B.sx[nt][sj][0], acc[m][nt][2]);
                    acc[m][nt][3] = fmaf(cs[nt][3], fsb * B.sx[nt][sj][1], acc[m][nt][3]);
                }
            }
        }
    }
}

__device__ __forceinline__ float bf16r(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

// SwiGLU of architecture.py:733-741 on bf16-rounded GEMM outputs
__device__ __forceinline__ float swiglu(float gv, float uv, float limit) {
    float gt = bf16r(gv), up = bf16r(uv);
    if (limit > 0.f) {
        up = fminf(fmaxf(up, -limit), limit);
        gt = fminf(gt, limit);
    }
    const float silu = gt / (1.0f + expf(-gt));
    return silu * up;
}

// Generic consumer loop.  `epi(it, red, tid)` runs on the 256 consumer
// threads after the fixed-order cross-warp reduction inputs are in `red`.
template <typename Decode, typename RowPtr, typename PreqScale, typename FP8Scale, typename Epi>
__device__ void consume(const Smem &sm, int i0, int i1, int ue8m0, int *err, long long lim, Decode decode,
                        RowPtr rowptr, PreqScale preq_scale, FP8Scale f8s, Epi epi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int g = lane >> 2, tig = lane & 3;
    volatile int *abort = sm.flags();
    float *red = sm.red();
    BRegs B;
    int key_src = -1, key_tok0 = -1, key_ntok = -1, key_a = -1;
    int q = 0;
    for (int i = i0; i < i1; ++i, ++q) {
        const Item it = decode(i);
        const int s = q % NSLOT;
        if (it.bsrc != key_src || it.tok0 != key_tok0 || it.ntok != key_ntok || it.a != key_a) {
            load_b(it, warp, lane, ue8m0, B, rowptr, preq_scale);
            key_src = it.bsrc; key_tok0 = it.tok0; key_ntok = it.ntok; key_a = it.a;
        }
        bool ok = !*abort;
        if (ok && !wf_wait(sm.full(s), (q / NSLOT) & 1, err, lim)) { *abort = 1; ok = false; }
        float acc[2][NTM][4];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int nt = 0; nt < NTM; ++nt)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[m][nt][c] = 0.f;
        if (ok) compute_item(it, sm.slot(s), warp, lane, B, acc, f8s);
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.empty(s));
        // partials -> red[warp][arow][tok]
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int nt = 0; nt < NTM; ++nt) {
                float *r0 = red + (warp * MAXR + 16 * m + g) * TPI + nt * 8 + 2 * tig;
                float *r1 = r0 + 8 * TPI;
                r0[0] = acc[m][nt][0]; r0[1] = acc[m][nt][1];
                r1[0] = acc[m][nt][2]; r1[1] = acc[m][nt][3];
            }
        bar_sync(1, NCT);
        epi(it, red, tid);
        bar_sync(1, NCT);
    }
}

__device__ __forceinline__ float red_sum(const float *red, int arow, int tok) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) v += red[(w * MAXR + arow) * TPI + tok];
    return v;
}

// ---------------------------------------------------------------------------
// router (K1, consumer warps)
// ---------------------------------------------------------------------------
constexpr int RKE = 2;  // 8-element chunks of a lane per gate row and K-eighth (D <= 4096)

// The gate weights a consumer warp multiplies in router pass p: K-eighth `warp`
// of the pass's two rows, as raw bf16 pairs.
struct GateChunk {
    uint4 w[2][RKE];
};

__device__ __forceinline__ GateChunk load_gate_chunk(const MoeArgs &a, int p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int nrows = (blockIdx.x < a.E) ? cdiv(a.E - blockIdx.x, G) : 0;
    const int eighth = a.D / 8;
    GateChunk c;
#pragma unroll
    for (int rl = 0; rl < 2; ++rl) {
        const int r = p + rl;
        const bool rv = r < nrows;
        const __nv_bfloat16 *wrow = a.gate_w + (size_t)(rv ? blockIdx.x + r * G : 0) * a.D + warp * eighth;
#pragma unroll
        for (int u = 0; u < RKE; ++u) {
            const int k = lane * 8 + u * 256;
            c.w[rl][u] = (rv && k < eighth) ? ldg128(wrow + k) : make_uint4(0, 0, 0, 0);
        }
    }
    return c;
}

// Router logits, logits[t][e] = sum_k x[t][k] w[e][k] (Gate.forward's linear,
// architecture.py:696-700): CTA b takes the rows e = b, b + G, ...; a pass covers
// two rows and up to RTP tokens; warp w the K-eighth [w D/8, (w+1) D/8) of both
// rows.  bf16 products are exact in fp64 and summed in fp64 (lane, then warp
// shuffle tree, then the eight warps in order), rounded once to fp32.  The gate
// weights are held in fp64, so each token element is converted once for both
// rows.  w0: the chunk of pass 0, loaded by the caller (before the launch's
// wait for the previous kernel: the gate weights do not depend on it).
// SMEM: the tokens are staged in shared memory at xsm (else read from a.x).
template <int RTP, bool SMEM>
__device__ void router_logits_t(const MoeArgs &a, const Smem &sm, const __nv_bfloat16 *xsm, const GateChunk &w0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = a.E, D = a.D, T = a.T;
    const int G = gridDim.x;
    static_assert(2 * NCW * RTP * 8 <= MISC_BYTES, "router partials must fit the misc buffer");
    double *part = sm.misc();  // [2 rows][NCW warps][RTP tokens]
    const int nrows = (blockIdx.x < E) ? cdiv(E - blockIdx.x, G) : 0;
    const int eighth = D / 8;
    for (int p = 0; p < nrows; p += 2) {
        double wd[2][RKE][8];
        {
            const GateChunk wc = p == 0 ? w0 : load_gate_chunk(a, p);
#pragma unroll
            for (int rl = 0; rl < 2; ++rl)
#pragma unroll
                for (int u = 0; u < RKE; ++u) {
                    const uint32_t wv[4] = {wc.w[rl][u].x, wc.w[rl][u].y, wc.w[rl][u].z, wc.w[rl][u].w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        wd[rl][u][2 * c] = (double)bf16_bits_to_f32(wv[c] & 0xffffu);
                        wd[rl][u][2 * c + 1] = (double)bf16_bits_to_f32(wv[c] >> 16);
                    }
                }
        }
        for (int t0 = 0; t0 < T; t0 += RTP) {
            const int nt = min(RTP, T - t0);
            auto load_x = [&](int t, int u) -> uint4 {
                const int k = lane * 8 + u * 256;
                const size_t off = (size_t)(t0 + t) * D + warp * eighth + k;
                return (t < nt && k < eighth) ? (SMEM ? lds128(xsm + off) : ldg128(a.x + off)) : make_uint4(0, 0, 0, 0);
            };
            // from global memory every load of the pass is issued before the first
            // use (one memory latency per pass: the critical path is latency, not
            // bytes); from shared memory each token's loads come with its math
            uint4 xg[SMEM ? 1 : RTP][RKE];
            if (!SMEM) {
#pragma unroll
                for (int t = 0; t < (SMEM ? 1 : RTP); ++t)
#pragma unroll
                    for (int u = 0; u < RKE; ++u) xg[t][u] = load_x(t, u);
            }
            double acc[2][RTP];
            if constexpr (RTP >= 8) {
                // eight staged tokens: each token's two row chains in turn (measured
                // faster here than interleaving all sixteen)
#pragma unroll
                for (int t = 0; t < RTP; ++t) {
                    acc[0][t] = 0.0;
                    acc[1][t] = 0.0;
                    if (t >= nt) continue;
#pragma unroll
                    for (int u = 0; u < RKE; ++u) {
                        const uint4 xq = SMEM ? load_x(t, u) : xg[SMEM ? 0 : t][u];
                        const uint32_t xv[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const double x0 = (double)bf16_bits_to_f32(xv[c] & 0xffffu);
                            const double x1 = (double)bf16_bits_to_f32(xv[c] >> 16);
                            acc[0][t] = fma(x0, wd[0][u][2 * c], acc[0][t]);
                            acc[1][t] = fma(x0, wd[1][u][2 * c], acc[1][t]);
                            acc[0][t] = fma(x1, wd[0][u][2 * c + 1], acc[0][t]);
                            acc[1][t] = fma(x1, wd[1][u][2 * c + 1], acc[1][t]);
                        }
                    }
                }
            } else {
                // four tokens from global memory: 16 independent fp64 chains per lane, NS sub-sums
                // for each of the two rows and RTP tokens (element e of the lane's
                // chunk goes to sub-sum e % NS), added in order at the end; masked
                // tokens multiply zeros
                constexpr int NS = 8 / RTP;
                double acc3[2][RTP][NS];
#pragma unroll
                for (int rl = 0; rl < 2; ++rl)
#pragma unroll
                    for (int t = 0; t < RTP; ++t)
#pragma unroll
                        for (int q = 0; q < NS; ++q) acc3[rl][t][q] = 0.0;
#pragma unroll
                for (int u = 0; u < RKE; ++u) {
                    uint32_t xv[RTP][4];
#pragma unroll
                    for (int t = 0; t < RTP; ++t) {
                        const uint4 xq = SMEM ? load_x(t, u) : xg[SMEM ? 0 : t][u];
                        xv[t][0] = xq.x; xv[t][1] = xq.y; xv[t][2] = xq.z; xv[t][3] = xq.w;
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
                            const int q = ((u * 4 + c) * 2 + hh) % NS;
#pragma unroll
                            for (int t = 0; t < RTP; ++t) {
                                const double xd = (double)bf16_bits_to_f32(hh ? (xv[t][c] >> 16) : (xv[t][c] & 0xffffu));
                                acc3[0][t][q] = fma(xd, wd[0][u][2 * c + hh], acc3[0][t][q]);
                                acc3[1][t][q] = fma(xd, wd[1][u][2 * c + hh], acc3[1][t][q]);
                            }
                        }
                }
#pragma unroll
                for (int rl = 0; rl < 2; ++rl)
#pragma unroll
                    for (int t = 0; t < RTP; ++t) {
                        double v = acc3[rl][t][0];
#pragma unroll
                        for (int q = 1; q < NS; ++q) v += acc3[rl][t][q];
                        acc[rl][t] = v;
                    }
            }
#pragma unroll
            for (int t = 0; t < RTP; ++t) {
                if (t >= nt) continue;
#pragma unroll
                for (int rl = 0; rl < 2; ++rl) {
                    double v = acc[rl][t];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    acc[rl][t] = v;
                }
            }
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < RTP; ++t)
#pragma unroll
                    for (int rl = 0; rl < 2; ++rl) part[(rl * NCW + warp) * RTP + t] = acc[rl][t];
            }
            bar_sync(1, NCT);
            if (threadIdx.x < 2 * RTP) {
                const int rl2 = threadIdx.x / RTP, t = threadIdx.x % RTP;
                const int r2 = p + rl2;
                if (r2 < nrows && t < nt) {
                    double v = 0.0;
#pragma unroll
                    for (int w = 0; w < NCW; ++w) v += part[(rl2 * NCW + w) * RTP + t];
                    a.logits[(size_t)(t0 + t) * E + blockIdx.x + r2 * G] = (float)v;
                }
            }
            bar_sync(1, NCT);
        }
    }
}

__device__ void router_logits(const MoeArgs &a, const Smem &sm, const __nv_bfloat16 *xsm, const GateChunk &w0) {
    // tokens in shared memory: eight per pass (loads are cheap, fewer barriers);
    // from global memory: four, every load of the pass in flight at once
    if (xsm) router_logits_t<8, true>(a, sm, xsm, w0);
    else router_logits_t<4, false>(a, sm, xsm, w0);
}

__device__ __forceinline__ void warp_argmax(float &v, int &idx) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
}

// Inclusive block scan (NCT threads) of a 64-bit value whose 16-bit fields add
// independently; `tot` receives the block total.  `ws` holds NCW words.
__device__ __forceinline__ unsigned long long block_scan_u64(unsigned long long v, unsigned long long *ws,
                                                             unsigned long long &tot) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) ws[warp] = v;
    bar_sync(1, NCT);
    unsigned long long before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < NCW; ++w) {
        const unsigned long long x = ws[w];
        if (w < warp) before += x;
        all += x;
    }
    bar_sync(1, NCT);
    tot = all;
    return v + before;
}

// Top-k of token t by one warp (Gate.forward, architecture.py:696-718): scores,
// + bias for the choice, K rounds of warp argmax (lowest index on ties),
// weights from the unbiased scores normalized in slot order (non-softmax)
// times route_scale.  NE experts per lane; rolled loops keep the code small,
// since it runs once per launch on a cold instruction cache.
// dry: a warm-up pass on whatever the logits hold (shared-memory outputs only,
// no global writes, no error reports) that loads this code into the SM's
// instruction cache before the real pass runs on the last router CTA.
// The routing inputs of topk_token, passed by value: inside the non-inlined
// function the kernel's argument block would be read through a pointer, one
// dependent load per field on a cold SM.
struct TopkIn {
    const float *logits;
    const float *gate_b;
    const long long *ids;
    const int *tid2eid;
    float *out_w;
    long long *out_idx;
    int *err;
    int E, K, score_func, hash;
    long long vocab;
    float route_scale;
};

__device__ __forceinline__ TopkIn topk_in(const MoeArgs &a) {
    TopkIn q;
    q.logits = a.logits; q.gate_b = a.gate_b; q.ids = a.ids; q.tid2eid = a.tid2eid;
    q.out_w = a.out_w; q.out_idx = a.out_idx; q.err = a.err;
    q.E = a.E; q.K = a.topk; q.score_func = a.score_func; q.hash = a.hash; q.vocab = a.vocab;
    q.route_scale = a.route_scale;
    return q;
}

template <int NE>
__device__ __noinline__ void topk_token(const TopkIn a, int t, int lane, float *sc_w, int16_t *ridx_s,
                                        int16_t *pof_s, float *rw_s, bool dry) {
    const int E = a.E, K = a.K;
    float sc[NE], bs[NE], gb[NE];
    // logits and gate bias in one round trip
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        const int e = lane + 32 * i;
        sc[i] = e < E ? __ldcg(a.logits + (size_t)t * E + e) : -INFINITY;
        gb[i] = (e < E && a.gate_b) ? __ldg(a.gate_b + e) : 0.f;
    }
    if (a.score_func == WF_SCORE_SOFTMAX) {
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < NE; ++i) mx = fmaxf(mx, sc[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            const int e = lane + 32 * i;
            sc[i] = e < E ? expf(sc[i] - mx) : 0.f;
            sum += sc[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
        for (int i = 0; i < NE; ++i) sc[i] = sc[i] / sum;
    } else if (a.score_func == WF_SCORE_SIGMOID) {
#pragma unroll
        for (int i = 0; i < NE; ++i) sc[i] = 1.0f / (1.0f + expf(-sc[i]));
    } else {
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            const float l = sc[i];
            sc[i] = sqrtf(l > 20.f ? l : log1pf(expf(l)));
        }
    }
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        const int e = lane + 32 * i;
        bs[i] = e < E ? (a.gate_b ? sc[i] + gb[i] : sc[i]) : -INFINITY;
        if (e < E) sc_w[e] = sc[i];
    }
    long long id = 0;
    if (a.hash) {
        id = __ldg(a.ids + t);
        if (id < 0 || id >= a.vocab) { if (lane == 0 && !dry) atomicOr(a.err, kErrExpertId); id = 0; }
    }
    if (a.hash) {
#pragma unroll 1
        for (int j = 0; j < K; ++j) {
            int ej = __ldg(a.tid2eid + id * K + j);
            if (ej < 0 || ej >= E) { if (lane == 0 && !dry) atomicOr(a.err, kErrExpertId); ej = 0; }
            if (lane == 0) ridx_s[t * K + j] = (int16_t)ej;
        }
    } else {
        // Biased scores as unsigned keys with the float order (+0 for -0, so equal
        // scores give equal keys); 0 marks an expert that is taken or absent.  Each
        // round takes the largest key, the lowest expert id among equal keys (torch
        // topk order), with two warp reductions; only the winning lane rescans its
        // candidates.
        uint32_t key[NE];
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            uint32_t u = __float_as_uint(bs[i] + 0.0f);
            u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            key[i] = (lane + 32 * i < E) ? u : 0u;
        }
        auto best = [&](uint32_t &bk, int &be) {
            bk = key[0];
            be = lane;
#pragma unroll
            for (int i = 1; i < NE; ++i)
                if (key[i] > bk) { bk = key[i]; be = lane + 32 * i; }  // ties keep the lower id
        };
        uint32_t bk;
        int be;
        best(bk, be);
#pragma unroll 1
        for (int j = 0; j < K; ++j) {
            const uint32_t m = __reduce_max_sync(0xffffffffu, bk);
            const int w = (int)__reduce_min_sync(0xffffffffu, bk == m ? (uint32_t)be : 0xffffffffu);
            const int ej = (w >= 0 && w < E) ? w : 0;  // a dry pass may see any bits
            if (be == w) {
#pragma unroll
                for (int i = 0; i < NE; ++i)
                    if (lane + 32 * i == w) key[i] = 0u;
                best(bk, be);
            }
            if (lane == 0) ridx_s[t * K + j] = (int16_t)ej;
        }
    }
    __syncwarp();
    float wj = 0.f;
    int ej = 0;
    if (lane < K) {
        ej = ridx_s[t * K + lane];
        wj = sc_w[ej];
    }
    float wsum = 0.f;
    for (int j = 0; j < K; ++j) wsum += __shfl_sync(0xffffffffu, wj, j);
    if (lane < K) {
        float w = wj;
        if (a.score_func != WF_SCORE_SOFTMAX) w = w / wsum;
        w = w * a.route_scale;
        rw_s[t * K + lane] = w;
        pof_s[t * K + lane] = -1;
        if (!dry && a.out_w) a.out_w[(size_t)t * K + lane] = w;
        if (!dry && a.out_idx) a.out_idx[(size_t)t * K + lane] = ej;
    }
    __syncwarp();
}

// Waits (bounded by `limit` SM cycles) until *ctr >= target, reading it with
// acquire semantics; on a timeout sets kErrTimeout and returns false.
__device__ bool wait_count(const unsigned *ctr, unsigned target, int *err, long long limit) {
    const long long t0 = clock64();
    while (true) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v >= target) return true;
        if (clock64() - t0 > limit) {
            atomicOr(err, kErrTimeout);
            return false;
        }
        __nanosleep(64);
    }
}

// Top-k of more tokens than one CTA has warps: router CTA b < ntk takes the
// tokens b * NCW + warp (+ ntk * NCW ...), one warp per token, once every router
// CTA's logits are written, and stores each token's experts and weights in
// a.ridx / a.rw for the CTA that builds the dispatch tables.
__device__ void topk_spread(const MoeArgs &a, const Smem &sm, unsigned nrc, unsigned ntk) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.topk;
    int16_t *ridx_s = reinterpret_cast<int16_t *>(sm.red());
    int16_t *pof_s = ridx_s + MAX_T * MAX_K;
    float *rw_s = reinterpret_cast<float *>(pof_s + MAX_T * MAX_K);
    float *sc_all = reinterpret_cast<float *>(sm.base + OFF_ROUTE);
    if (threadIdx.x == 0) wait_count(a.cnt_router, nrc, a.err, a.wait_limit);
    bar_sync(1, NCT);
    for (int t = (int)blockIdx.x * NCW + warp; t < a.T; t += (int)ntk * NCW) {
        if (a.E <= 256) topk_token<8>(topk_in(a), t, lane, sc_all + warp * MAX_E, ridx_s, pof_s, rw_s, false);
        else topk_token<MAX_E / 32>(topk_in(a), t, lane, sc_all + warp * MAX_E, ridx_s, pof_s, rw_s, false);
        if (lane < K) {
            a.ridx[t * K + lane] = ridx_s[t * K + lane];
            a.rw[t * K + lane] = rw_s[t * K + lane];
        }
    }
    __threadfence();
    bar_sync(1, NCT);
}

// Top-k and dispatch tables; run by the 256 consumer threads of one CTA.
// Every phase is spread over the block (the router kernel's critical path):
//   1. top-k per token, one warp per token           -> ridx_s, rw_s, outputs
//   2. per (token, slot): keep flag (a duplicate keeps its last slot), expert
//      counts and per-expert token bitmaps (shared-memory atomics)
//   3. block scan over local experts                 -> act_* tables, header
//   4. per kept slot: rank among the expert's tokens (bitmap popcount) -> pair
//   5. per token: its pairs in ascending expert order -> tok_pairs
__device__ void topk_dispatch(const MoeArgs &a, const Smem &sm, bool spread = false) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int T = a.T, E = a.E, K = a.topk, El = a.El;
    static_assert(MAX_T * MAX_K * (2 + 2 + 4) <= RED_BYTES, "top-k tables must fit the reduction buffer");
    static_assert(MAX_E * 4 <= MISC_BYTES, "expert counts must fit the misc buffer");
    static_assert(TOPK_ROUTE_BYTES <= ROUTE_BYTES, "token bitmaps must fit the route buffer");
    int16_t *ridx_s = reinterpret_cast<int16_t *>(sm.red());          // [T*K] expert
    int16_t *pof_s = ridx_s + MAX_T * MAX_K;                            // [T*K] pair or -1
    float *rw_s = reinterpret_cast<float *>(pof_s + MAX_T * MAX_K);     // [T*K] weight
    int *cnt_s = reinterpret_cast<int *>(sm.misc());                    // [El]
    uint32_t *bm = reinterpret_cast<uint32_t *>(sm.base + OFF_ROUTE);   // [El][TW]
    int *off_s = reinterpret_cast<int *>(bm + MAX_E * (MAX_T / 32));    // [El]
    unsigned long long *scan_ws = reinterpret_cast<unsigned long long *>(off_s + MAX_E);   // [NCW]
    const int TW = (T + 31) >> 5;
    // ---- 1. top-k: one warp per token, scores of the warp's token in shared memory
    // (routed-only calls take the routing computed by the ranks that own the tokens;
    // `spread`: the router CTAs computed it, topk_spread, into a.ridx / a.rw)
    if (a.given || spread) {
        for (int slot = tid; slot < T * K; slot += NCT) {
            long long e = a.given ? __ldg(a.in_idx + slot) : (long long)__ldcg(a.ridx + slot);
            if (e < 0 || e >= E) { atomicOr(a.err, kErrExpertId); e = 0; }
            ridx_s[slot] = (int16_t)e;
            rw_s[slot] = a.given ? __ldg(a.in_w + slot) : __ldcg(a.rw + slot);
            pof_s[slot] = -1;
        }
    } else {
        float *sc_all = reinterpret_cast<float *>(sm.base + OFF_ROUTE);  // [NCW][MAX_E]
        for (int t = warp; t < T; t += NCW) {
            if (E <= 256) topk_token<8>(topk_in(a), t, lane, sc_all + warp * MAX_E, ridx_s, pof_s, rw_s, false);
            else topk_token<MAX_E / 32>(topk_in(a), t, lane, sc_all + warp * MAX_E, ridx_s, pof_s, rw_s, false);
        }
    }
    bar_sync(1, NCT);
    if (a.route_only) {
        __threadfence();
        return;
    }
    for (int i = tid; i < El; i += NCT) cnt_s[i] = 0;
    for (int i = tid; i < El * TW; i += NCT) bm[i] = 0u;
    bar_sync(1, NCT);
    // ---- 2. keep flags, counts, bitmaps
    for (int slot = tid; slot < T * K; slot += NCT) {
        const int t = slot / K, j = slot - t * K;
        const int e = ridx_s[slot];
        bool later = false;
        for (int j2 = j + 1; j2 < K; ++j2) later |= ridx_s[t * K + j2] == e;
        const int el = e - a.e0;
        if (!later && el >= 0 && el < El) {
            pof_s[slot] = -2;
            atomicAdd(cnt_s + el, 1);
            atomicOr(bm + el * TW + (t >> 5), 1u << (t & 31));
        }
    }
    bar_sync(1, NCT);
    // ---- 3. scan over local experts (two per thread): pair offset, item offsets, active index
    const int per2 = a.I / a.g.nh13, per3 = a.D / a.g.r2;
    int c0 = 0, c1 = 0;
    const int el0 = 2 * tid, el1 = 2 * tid + 1;
    if (el0 < El) c0 = cnt_s[el0];
    if (el1 < El) c1 = cnt_s[el1];
    auto pack = [](int c) -> unsigned long long {
        return (unsigned long long)c | ((unsigned long long)cdiv(c, TPI) << 16) |
               ((unsigned long long)(c > 0) << 32);
    };
    const unsigned long long v0 = pack(c0), v1 = pack(c1);
    unsigned long long tot;
    const unsigned long long inc = block_scan_u64(v0 + v1, scan_ws, tot);
    unsigned long long ex0 = inc - v0 - v1;
    auto emit = [&](int el, int c, unsigned long long ex) {
        if (el >= El) return;
        const int off = (int)(ex & 0xffff), tg = (int)((ex >> 16) & 0xffff), n = (int)((ex >> 32) & 0xffff);
        off_s[el] = off;
        if (c) {
            a.act_expert[n] = a.e0 + el;
            a.act_off[n] = off;
            a.act_it2[n] = per2 * tg;
            a.act_it3[n] = per3 * tg;
        }
    };
    emit(el0, c0, ex0);
    emit(el1, c1, ex0 + v0);
    if (tid == NCT - 1) {
        const int off = (int)(tot & 0xffff), tg = (int)((tot >> 16) & 0xffff), n = (int)((tot >> 32) & 0xffff);
        a.act_off[n] = off; a.act_it2[n] = per2 * tg; a.act_it3[n] = per3 * tg;
        a.hdr[H_NACT] = n; a.hdr[H_IT2] = per2 * tg; a.hdr[H_IT3] = per3 * tg; a.hdr[H_TGT] = tg;
        a.hdr[H_NPAIR] = off;
    }
    bar_sync(1, NCT);
    // ---- 4. pairs: expert ascending, token ascending within an expert.  On the
    // tcgen05 engine each slot's expert and pair (-1: none) go to a.ridx and
    // a.tok_pairs, and the w2 kernel builds the per-token lists of step 5 in its
    // prologue, while the w1/w3 kernel runs.
    for (int slot = tid; slot < T * K; slot += NCT) {
        if (a.tc) a.ridx[slot] = ridx_s[slot];
        if (pof_s[slot] != -2) {
            if (a.tc) a.tok_pairs[slot] = -1;
            continue;
        }
        const int t = slot / K;
        const int el = ridx_s[slot] - a.e0;
        const uint32_t *row = bm + el * TW;
        int rank = __popc(row[t >> 5] & ((1u << (t & 31)) - 1u));
        for (int w = 0; w < (t >> 5); ++w) rank += __popc(row[w]);
        const int p = off_s[el] + rank;
        a.pair_tok[p] = t;
        a.pair_w[p] = rw_s[slot];
        pof_s[slot] = (int16_t)p;
        if (a.tc) a.tok_pairs[slot] = p;
    }
    if (a.tc) {
        __threadfence();
        return;
    }
    bar_sync(1, NCT);
    // ---- 5. each token's pairs in ascending expert order (a token's kept experts
    // are distinct, so a slot's place is the number of its kept slots with a
    // smaller expert)
    for (int t = tid; t < T; t += NCT) {
        int n = 0;
        for (int j = 0; j < K; ++j) {
            const int p = pof_s[t * K + j];
            if (p < 0) continue;
            const int e = ridx_s[t * K + j];
            int rank = 0;
            for (int j2 = 0; j2 < K; ++j2)
                rank += (pof_s[t * K + j2] >= 0 && ridx_s[t * K + j2] < e) ? 1 : 0;
            a.tok_pairs[t * K + rank] = p;
            ++n;
        }
        a.tok_np[t] = n;
    }
    __threadfence();
}

// ---------------------------------------------------------------------------
// combine of one output row block (K3): ascending-expert fp32 sum + shared
// ---------------------------------------------------------------------------
template <int NTH = NCT>
__device__ void combine_rows(const MoeArgs &a, int row0, int nrows) {
    const int T = a.T, D = a.D, K = a.topk;
    const unsigned short *o = reinterpret_cast<const unsigned short *>(a.o);
    const unsigned short *os = reinterpret_cast<const unsigned short *>(a.os);
    for (int idx = threadIdx.x; idx < T * nrows; idx += NTH) {
        const int t = idx / nrows, r = row0 + idx % nrows;
        float acc = 0.f;
        const int np = __ldcg(a.tok_np + t);
        for (int qq = 0; qq < np; ++qq) {
            const int p = __ldcg(a.tok_pairs + t * K + qq);
            acc += bf16_bits_to_f32(__ldcg(o + (size_t)p * D + r));
        }
        if (a.sh_add && t >= a.sh0 && t < a.sh0 + a.shT) acc += bf16_bits_to_f32(__ldcg(os + (size_t)t * D + r));
        if (a.partial) a.y_partial[(size_t)t * D + r] = acc;
        else a.y[(size_t)t * D + r] = __float2bfloat16_rn(acc);
    }
}

// combine_rows with 8 consecutive rows of one token per item (16-byte loads and
// stores) and two items per thread whose pair lists and pair rows are all
// loaded before the first add; same fp32 sum in the same order.  nrows and
// row0 are multiples of 8.  With np_s / tp_s (a shared-memory copy of tok_np
// and tok_pairs) the pair lists cost no global round trip.
template <int NTH>
__device__ void combine_rows_v8(const MoeArgs &a, int row0, int nrows, const uint8_t *np_s = nullptr,
                                const int16_t *tp_s = nullptr) {
    const int T = a.T, D = a.D, K = a.topk, nv = nrows / 8, n = T * nv;
    for (int base = threadIdx.x; base < n; base += 2 * NTH) {
        int tt[2], rr[2], np[2], pr[2][MAX_K];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int idx = base + j * NTH;
            const bool ok = idx < n;
            tt[j] = ok ? idx / nv : 0;
            rr[j] = row0 + 8 * (ok ? idx - tt[j] * nv : 0);
            if (np_s) {
                np[j] = ok ? np_s[tt[j]] : 0;
#pragma unroll
                for (int q = 0; q < MAX_K; ++q) pr[j][q] = (ok && q < K) ? tp_s[tt[j] * K + q] : 0;
            } else {
                np[j] = ok ? __ldcg(a.tok_np + tt[j]) : 0;
#pragma unroll
                for (int q = 0; q < MAX_K; ++q) pr[j][q] = (ok && q < K) ? __ldcg(a.tok_pairs + tt[j] * K + q) : 0;
            }
        }
        uint4 v[2][MAX_K];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int q = 0; q < MAX_K; ++q)
                v[j][q] = q < np[j] ? ldcg128(a.o + (size_t)pr[j][q] * D + rr[j]) : make_uint4(0, 0, 0, 0);
        uint4 sv[2];
#pragma unroll
        for (int j = 0; j < 2; ++j)
            sv[j] = (a.sh_add && base + j * NTH < n && tt[j] >= a.sh0 && tt[j] < a.sh0 + a.shT)
                        ? ldcg128(a.os + (size_t)tt[j] * D + rr[j])
                        : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            if (base + j * NTH >= n) continue;
            float acc[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
            for (int q = 0; q < MAX_K; ++q) {
                if (q >= np[j]) break;
                const uint32_t u[4] = {v[j][q].x, v[j][q].y, v[j][q].z, v[j][q].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    acc[2 * e] += bf16_bits_to_f32(u[e] & 0xffffu);
                    acc[2 * e + 1] += bf16_bits_to_f32(u[e] >> 16);
                }
            }
            const int t = tt[j], r = rr[j];
            if (a.partial) {
                if (a.sh_add && t >= a.sh0 && t < a.sh0 + a.shT) {
                    const uint32_t u[4] = {sv[j].x, sv[j].y, sv[j].z, sv[j].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[2 * e] += bf16_bits_to_f32(u[e] & 0xffffu);
                        acc[2 * e + 1] += bf16_bits_to_f32(u[e] >> 16);
                    }
                }
                // expert parallelism over peer memory: the row goes to its owner's
                // receive buffer, in this rank's slot
                const int o = a.ep ? t / a.Tr : 0;
                float *drow = a.ep ? a.ep_yrecv[o] + ((size_t)a.ep_rank * a.Tr + (t - o * a.Tr)) * D
                                   : a.y_partial + (size_t)t * D;
                float4 *dst = reinterpret_cast<float4 *>(drow + r);
                dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
            } else {
                const uint32_t u[4] = {sv[j].x, sv[j].y, sv[j].z, sv[j].w};
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float lo = acc[2 * e] + bf16_bits_to_f32(u[e] & 0xffffu);
                    const float hi = acc[2 * e + 1] + bf16_bits_to_f32(u[e] >> 16);
                    o[e] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
                           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
                }
                *reinterpret_cast<uint4 *>(a.y + (size_t)t * D + r) = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ void init_smem(const Smem &sm) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; ++s) {
            mbar_init(sm.full(s), 1);
            mbar_init(sm.empty(s), NCW);
        }
        sm.flags()[0] = 0;  // abort
        sm.flags()[1] = 0;  // scratch flag
        fence_mbar_init();
    }
    __syncthreads();
}

struct MoeRowPtr {
    const MoeArgs *a;
    const int16_t *pair_tok;  // shared-memory copy (K2)
    __device__ const void *operator()(const Item &it, int j) const {
        const int p = it.tok0 + j;
        switch (it.bsrc) {
            case BS_XPAIR: return a->x + (size_t)pair_tok[p] * a->D;
            case BS_XTOK: return a->x + (size_t)p * a->D;
            case BS_H: return a->h + (size_t)p * a->I;
            default: return a->hs + (size_t)p * a->I;
        }
    }
};

struct NoPreq {
    __device__ float operator()(const Item &, int, int) const { return 0.f; }
};

// act_quant (torch_ops.py:33-49) of the layer input for the tcgen05 expert
// phases, by one warp: token t by CTA t mod grid, eight 128-blocks per round
// (loads first), four elements per lane.  Scales are powers of two (ue8m0),
// stored as e8m0 bytes.
__device__ void quantize_tokens_warp(const MoeArgs &a) {
    const int lane = threadIdx.x & 31;
    const int nb = a.D / 128;
    for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
        for (int b0 = 0; b0 < nb; b0 += 8) {
            uint2 u[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int b = b0 + q;
                u[q] = b < nb ? __ldg(reinterpret_cast<const uint2 *>(a.x + (size_t)t * a.D + b * 128 + 4 * lane))
                              : make_uint2(0, 0);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int b = b0 + q;
                if (b >= nb) break;
                const float v0 = bf16_bits_to_f32(u[q].x & 0xffffu), v1 = bf16_bits_to_f32(u[q].x >> 16);
                const float v2 = bf16_bits_to_f32(u[q].y & 0xffffu), v3 = bf16_bits_to_f32(u[q].y >> 16);
                float m = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float s = round_scale_e8(fmaxf(m, 1e-4f), 1);
                const float inv = 1.0f / s;  // exact: s is a power of two
                auto qz = [&](float v) { return fminf(fmaxf(v * inv, -448.f), 448.f); };
                const uint32_t lo = f32x2_to_e4m3x2(qz(v0), qz(v1)), hi = f32x2_to_e4m3x2(qz(v2), qz(v3));
                *reinterpret_cast<uint32_t *>(a.xq + (size_t)t * a.D + b * 128 + 4 * lane) = lo | (hi << 16);
                if (lane == 0) a.xs[(size_t)t * nb + b] = (uint8_t)((__float_as_uint(s) >> 23) & 0xffu);
            }
        }
    }
}

__global__ void __launch_bounds__(NTHR, 1) k_moe_up(const __grid_constant__ MoeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem sm{smem_raw};
    // the first pass's gate rows do not depend on the previous kernel
    GateChunk w0{};
    if (!a.given && (threadIdx.x >> 5) < NCW) w0 = load_gate_chunk(a, 0);
    init_smem(sm);
    pdl_wait();
    pdl_launch_dependents();
    const bool given = a.given;
    const int n = (a.route_only || a.tc) ? 0 : (a.I / a.g.nhs13) * cdiv(a.shT, TPI);
    int i0, i1;
    item_range(n, i0, i1);
    auto decode = [&](int i) { return decode_moe(KID_UP, a, i, 0, 0, nullptr, nullptr, nullptr); };
    // tcgen05 mode: the ring is idle, so up to TPI token rows are staged in it with
    // one bulk copy for the router, and the producer warp quantizes the tokens
    const size_t xbytes = (size_t)a.T * a.D * 2;
    const bool stage_x = a.tc && !given && a.T <= TPI && xbytes + 8192 <= (size_t)NSLOT * SLOT_BYTES &&
                         blockIdx.x < (unsigned)a.E;
    if ((threadIdx.x >> 5) == NCW) {
        if (a.tc) {
            if (stage_x && (threadIdx.x & 31) == 0) {
                mbar_arrive_expect_tx(sm.full(0), (uint32_t)xbytes);
                bulk_g2s(sm.slot(0), a.x, (uint32_t)xbytes, sm.full(0));
            }
            if (!a.route_only) quantize_tokens_warp(a);
            if (!given) {
                // warm the top-k code on this SM (the last router CTA runs it for real)
                uint8_t *scratch = sm.slot(0) + (size_t)NSLOT * SLOT_BYTES - 8192;
                float *sc_w = reinterpret_cast<float *>(scratch);                    // [MAX_E]
                int16_t *ri = reinterpret_cast<int16_t *>(scratch + 4 * MAX_E);        // [MAX_K]
                int16_t *po = ri + MAX_K;                                              // [MAX_K]
                float *rw = reinterpret_cast<float *>(po + MAX_K);                     // [MAX_K]
                if (a.E <= 256) topk_token<8>(topk_in(a), 0, threadIdx.x & 31, sc_w, ri, po, rw, true);
                else topk_token<MAX_E / 32>(topk_in(a), 0, threadIdx.x & 31, sc_w, ri, po, rw, true);
            }
            return;
        }
        produce(sm, i0, i1, a.err, a.wait_limit, decode);
        return;
    }
    if (given) {
        // routing given: no router; CTA 0 builds the dispatch tables
        if (blockIdx.x == 0) topk_dispatch(a, sm);
    } else {
    const __nv_bfloat16 *xsm = nullptr;
    if (stage_x && wf_wait(sm.full(0), 0, a.err)) xsm = reinterpret_cast<const __nv_bfloat16 *>(sm.slot(0));
    router_logits(a, sm, xsm, w0);
    __threadfence();
    bar_sync(1, NCT);
    const unsigned nrc = min((unsigned)a.E, gridDim.x);
    if (blockIdx.x < nrc) {
        // More tokens than warps: the top-k runs on the first ntk router CTAs, one
        // warp per token, and the last of them to finish builds the tables.
        // Otherwise the last router CTA to arrive does both.
        const bool spread = a.T > NCW;
        const unsigned ntk = spread ? min(nrc, (unsigned)cdiv(a.T, NCW)) : 1u;
        if (threadIdx.x == 0) {
            const unsigned old = atomicAdd(a.cnt_router, 1u);
            sm.flags()[1] = spread ? (blockIdx.x < ntk) : (old == nrc - 1);
        }
        bar_sync(1, NCT);
        if (sm.flags()[1]) {
            if (spread) {
                topk_spread(a, sm, nrc, ntk);
                if (threadIdx.x == 0) {
                    const unsigned old = atomicAdd(a.cnt_router + 1, 1u);
                    sm.flags()[1] = (old == ntk - 1);
                }
                bar_sync(1, NCT);
            }
            if (!spread || sm.flags()[1]) {
                __threadfence();
                topk_dispatch(a, sm, spread);
                if (threadIdx.x == 0) { a.cnt_router[0] = 0u; a.cnt_router[1] = 0u; }
            }
        }
        bar_sync(1, NCT);
    }
    }
    MoeRowPtr rp{&a, nullptr};
    auto f8 = [&](int rblk, int kb) {
        const int kbs = a.D / 128;
        if (a.shared_f32) return __ldg((const float *)a.ss13 + rblk * kbs + kb);
        return e8m0_to_f32(__ldg((const uint8_t *)a.ss13 + rblk * kbs + kb));
    };
    auto epi = [&](const Item &it, const float *red, int tid) {
        const int nh = it.rrows;
        for (int idx = tid; idx < nh * it.ntok; idx += NCT) {
            const int tok = idx / nh, j = idx % nh;
            const float hv = swiglu(red_sum(red, j, tok), red_sum(red, nh + j, tok), a.swiglu_limit);
            a.hs[(size_t)(it.tok0 + tok) * a.I + it.row0 + j] = __float2bfloat16_rn(hv);
        }
    };
    consume(sm, i0, i1, a.ue8m0, a.err, a.wait_limit, decode, rp, NoPreq{}, f8, epi);
}

__global__ void __launch_bounds__(NTHR, 1) k_moe_mid(const __grid_constant__ MoeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem sm{smem_raw};
    init_smem(sm);
    pdl_wait();
    pdl_launch_dependents();
    const int n_act = a.hdr[H_NACT], n_it2 = a.hdr[H_IT2];
    load_route(sm, a.act_expert, a.act_off, a.act_it2, a.pair_tok, a.pair_w, n_act, a.hdr[H_NPAIR]);
    const RouteSm rt = route_sm(sm);
    const int n = n_it2 + (a.D / a.g.rs2) * cdiv(a.shT, TPI);
    int i0, i1;
    item_range(n, i0, i1);
    auto decode = [&, c = Cursor{-1, 0}](int i) mutable {
        if (i < n_it2) {
            if (c.i < 0) c = cursor_at(rt, n_act, i);
            while (c.i < i) cursor_next(rt, n_act, c);
        }
        return decode_moe(KID_MID, a, i, c.ai, n_it2, rt.act_expert, rt.act_off, rt.act_it);
    };
    if ((threadIdx.x >> 5) == NCW) {
        produce(sm, i0, i1, a.err, a.wait_limit, decode);
        return;
    }
    MoeRowPtr rp{&a, rt.pair_tok};
    auto f8 = [&](int rblk, int kb) {
        const int kbs = a.I / 128;
        if (a.shared_f32) return __ldg((const float *)a.ss2 + rblk * kbs + kb);
        return e8m0_to_f32(__ldg((const uint8_t *)a.ss2 + rblk * kbs + kb));
    };
    auto epi = [&](const Item &it, const float *red, int tid) {
        if (it.ep == EP_RSWIGLU) {
            const int nh = it.rrows;
            for (int idx = tid; idx < nh * it.ntok; idx += NCT) {
                const int tok = idx / nh, j = idx % nh;
                const int p = it.tok0 + tok;
                float hv = swiglu(red_sum(red, j, tok), red_sum(red, nh + j, tok), a.swiglu_limit);
                hv = rt.pair_w[p] * hv;
                a.h[(size_t)p * a.I + it.row0 + j] = __float2bfloat16_rn(hv);
            }
        } else {
            const int nr = it.rrows;
            for (int idx = tid; idx < nr * it.ntok; idx += NCT) {
                const int tok = idx / nr, r = idx % nr;
                a.os[(size_t)(it.tok0 + tok) * a.D + it.row0 + r] =
                    __float2bfloat16_rn(red_sum(red, r, tok));
            }
        }
    };
    consume(sm, i0, i1, a.ue8m0, a.err, a.wait_limit, decode, rp, NoPreq{}, f8, epi);
}

__global__ void __launch_bounds__(NTHR, 1) k_moe_down(const __grid_constant__ MoeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem sm{smem_raw};
    init_smem(sm);
    pdl_wait();
    pdl_launch_dependents();
    const int n_act = a.hdr[H_NACT], n = a.hdr[H_IT3], tgt = a.hdr[H_TGT];
    if (n_act == 0) {  // no local expert has tokens: y = shared part only
        if ((threadIdx.x >> 5) == NCW) return;
        const int nrb = a.D / a.g.r2;
        for (int rb = blockIdx.x; rb < nrb; rb += gridDim.x) combine_rows(a, rb * a.g.r2, a.g.r2);
        return;
    }
    load_route(sm, a.act_expert, a.act_off, a.act_it3, a.pair_tok, a.pair_w, n_act, a.hdr[H_NPAIR]);
    const RouteSm rt = route_sm(sm);
    int i0, i1;
    item_range(n, i0, i1);
    auto decode = [&, c = Cursor{-1, 0}](int i) mutable {
        if (c.i < 0) c = cursor_at(rt, n_act, i);
        while (c.i < i) cursor_next(rt, n_act, c);
        return decode_moe(KID_DOWN, a, i, c.ai, 0, rt.act_expert, rt.act_off, rt.act_it);
    };
    if ((threadIdx.x >> 5) == NCW) {
        produce(sm, i0, i1, a.err, a.wait_limit, decode);
        return;
    }
    MoeRowPtr rp{&a, rt.pair_tok};
    auto f8 = [&](int, int) { return 0.f; };
    volatile int *flag = sm.flags() + 1;
    auto epi = [&](const Item &it, const float *red, int tid) {
        const int nr = it.rrows;
        for (int idx = tid; idx < nr * it.ntok; idx += NCT) {
            const int tok = idx / nr, r = idx % nr;
            a.o[(size_t)(it.tok0 + tok) * a.D + it.row0 + r] = __float2bfloat16_rn(red_sum(red, r, tok));
        }
        __threadfence();
        bar_sync(1, NCT);
        if (tid == 0) {
            const unsigned old = atomicAdd(a.cnt_rb + it.rb, 1u);
            *flag = (old == (unsigned)tgt - 1);
        }
        bar_sync(1, NCT);
        if (*flag) {
            __threadfence();
            combine_rows(a, it.row0, nr);
            if (tid == 0) a.cnt_rb[it.rb] = 0u;
        }
    };
    consume(sm, i0, i1, a.ue8m0, a.err, a.wait_limit, decode, rp, NoPreq{}, f8, epi);
}

__global__ void k_moe_finish(const float *yp, const __nv_bfloat16 *os, __nv_bfloat16 *y, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = __float2bfloat16_rn(yp[i] + __bfloat162float(os[i]));
}

// y[i] = bf16(parts[0][i] + parts[1][i] + ... + parts[P-1][i]), left to right
// (four consecutive elements per thread; n4 = n / 4)
__global__ void k_sum_ranks(const float4 *parts, int P, long long n4, uint2 *y) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        float4 acc = __ldg(parts + i);
        for (int p = 1; p < P; ++p) {
            const float4 v = __ldg(parts + (size_t)p * n4 + i);
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        const uint32_t lo = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc.x)) |
                            ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc.y)) << 16);
        const uint32_t hi = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc.z)) |
                            ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc.w)) << 16);
        y[i] = make_uint2(lo, hi);
    }
}

__global__ void k_to_bf16(const float *src, __nv_bfloat16 *dst, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

#include "wf_moe_tc.cuh"
#include "wf_moe_fused.cuh"

__global__ void __launch_bounds__(NTHR, 1) k_dense(const __grid_constant__ DenseArgs d) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem sm{smem_raw};
    init_smem(sm);
    const int n = d.nkc * (d.N / d.rows) * (d.G > 0 ? d.G : cdiv(d.M, TPI));
    int i0, i1;
    item_range(n, i0, i1);
    auto decode = [&](int i) { return decode_dense(d, i); };
    if ((threadIdx.x >> 5) == NCW) {
        produce(sm, i0, i1, d.err, kWaitLimitCycles, decode);
        return;
    }
    auto rowptr = [&](const Item &it, int j) -> const void * {
        return d.a + (size_t)(it.tok0 + j) * d.K + (size_t)it.kc * d.Kc;
    };
    auto preq = [&](const Item &it, int j, int s) {
        const size_t ix = (size_t)(it.tok0 + j) * (d.K / 128) + it.kb0 + s;
        return d.a_f32 ? __ldg((const float *)d.a_s + ix) : e8m0_to_f32(__ldg((const uint8_t *)d.a_s + ix));
    };
    auto f8 = [&](int rblk, int kb) {
        const size_t ix = (size_t)rblk * (d.K / 128) + kb;
        return d.b_f32 ? __ldg((const float *)d.b_s + ix) : e8m0_to_f32(__ldg((const uint8_t *)d.b_s + ix));
    };
    volatile int *flag = sm.flags() + 1;
    auto epi = [&](const Item &it, const float *red, int tid) {
        const int nr = it.rrows;
        const int M = d.G > 0 ? d.G : d.M;
        if (d.nkc == 1) {
            for (int idx = tid; idx < nr * it.ntok; idx += NCT) {
                const int tok = idx / nr, r = idx % nr;
                d.out[(size_t)(it.tok0 + tok) * d.N + it.row0 + r] = __float2bfloat16_rn(red_sum(red, r, tok));
            }
            return;
        }
        // split-K: fp32 partial per chunk; the last chunk to arrive sums them in chunk order
        for (int idx = tid; idx < nr * it.ntok; idx += NCT) {
            const int tok = idx / nr, r = idx % nr;
            d.part[((size_t)it.kc * M + it.tok0 + tok) * d.N + it.row0 + r] = red_sum(red, r, tok);
        }
        __threadfence();
        bar_sync(1, NCT);
        if (tid == 0) *flag = (atomicAdd(d.cnt + it.rb, 1u) == (unsigned)d.nkc - 1);
        bar_sync(1, NCT);
        if (*flag) {
            __threadfence();
            for (int idx = tid; idx < nr * it.ntok; idx += NCT) {
                const int tok = idx / nr, r = idx % nr;
                float v = 0.f;
                for (int c = 0; c < d.nkc; ++c)
                    v += __ldcg(d.part + ((size_t)c * M + it.tok0 + tok) * d.N + it.row0 + r);
                d.out[(size_t)(it.tok0 + tok) * d.N + it.row0 + r] = __float2bfloat16_rn(v);
            }
            if (tid == 0) d.cnt[it.rb] = 0u;
        }
    };
    consume(sm, i0, i1, 1, d.err, kWaitLimitCycles, decode, rowptr, preq, f8, epi);
}

// ---- standalone quantizers --------------------------------------------------
// act_quant: one warp per (row, 128-block); lane handles 4 elements.
__global__ void k_act_quant(const __nv_bfloat16 *x, long long M, long long K, int block,
                            int ue8m0, uint8_t *q, void *s, int s_f32) {
    const long long nb = K / block;
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= M * nb) return;
    const long long row = wid / nb, b = wid % nb;
    const __nv_bfloat16 *src = x + row * K + b * block;
    float amax = 0.f;
    for (int e = lane; e < block; e += 32) amax = fmaxf(amax, fabsf(__bfloat162float(src[e])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = round_scale_e8(fmaxf(amax, 1e-4f), ue8m0);
    for (int e = lane; e < block; e += 32) {
        float v = __bfloat162float(src[e]);
        v = ue8m0 ? v * (1.0f / sc) : __fdiv_rn(v, sc);
        v = fminf(fmaxf(v, -448.f), 448.f);
        q[row * K + b * block + e] = (uint8_t)(f32x2_to_e4m3x2(v, 0.f) & 0xff);
    }
    if (lane == 0) {
        if (s_f32) ((float *)s)[row * nb + b] = sc;
        else ((uint8_t *)s)[row * nb + b] = (uint8_t)((__float_as_uint(sc) >> 23) & 0xff);
    }
}

// fp4_act_quant: one thread per 32-block.  E2M1 code of |q| by the midpoint
// table with ties to the even code (torch_ops.py:52-58).
__device__ __forceinline__ uint32_t e2m1_code(float a) {
    const float mid[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
    int lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 7; ++i) { lo += mid[i] < a; hi += mid[i] <= a; }
    return (uint32_t)(lo + ((hi != lo) && (lo & 1)));
}

__global__ void k_fp4_act_quant(const __nv_bfloat16 *x, long long M, long long K, uint8_t *q,
                                uint8_t *s) {
    const long long nb = K / 32;
    const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= M * nb) return;
    const long long row = id / nb, b = id % nb;
    const __nv_bfloat16 *src = x + row * K + b * 32;
    float v[32];
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 32; ++e) { v[e] = __bfloat162float(src[e]); amax = fmaxf(amax, fabsf(v[e])); }
    amax = fmaxf(amax, 6.0f * 1.1754943508222875e-38f);
    const float x6 = amax * (1.0f / 6.0f);
    const uint32_t bits = __float_as_uint(x6);
    const float sc = (bits & 0x7fffffu) ? __uint_as_float(((bits >> 23) + 1) << 23) : x6;
    uint8_t *dst = q + row * (K / 2) + b * 16;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        float q0 = fminf(fmaxf(v[2 * e] / sc, -6.f), 6.f);
        float q1 = fminf(fmaxf(v[2 * e + 1] / sc, -6.f), 6.f);
        uint32_t c0 = e2m1_code(fabsf(q0)) | (q0 < 0.f ? 8u : 0u);
        uint32_t c1 = e2m1_code(fabsf(q1)) | (q1 < 0.f ? 8u : 0u);
        dst[e] = (uint8_t)(c0 | (c1 << 4));
    }
    s[row * nb + b] = (uint8_t)((__float_as_uint(sc) >> 23) & 0xff);
}

__global__ void k_scale_range(const uint8_t *s, long long n, int *bad) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const uint8_t b = s[i];
        if (b == 0 || b == 255) { atomicOr(bad, 1); return; }
    }
}

}  // namespace wf

// =============================================================================
// host side: C ABI
// =============================================================================
namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    return WF_E_CUDA;
}

struct DevInfo {
    int sms = 0;
    bool attr_done = false;
};
thread_local DevInfo g_dev[64];

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    DevInfo &d = g_dev[dev];
    if (!d.sms) cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    return d.sms;
}

int ensure_attrs() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return WF_E_CUDA;
    DevInfo &d = g_dev[dev];
    if (d.attr_done) return WF_OK;
    const void *ks[] = {(const void *)wf::k_moe_up, (const void *)wf::k_moe_mid,
                        (const void *)wf::k_moe_down, (const void *)wf::k_dense};
    for (const void *k : ks) {
        cudaError_t e =
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, wf::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    }
    const void *ts[] = {(const void *)wf::mtc::k_moe_tc<2>, (const void *)wf::mtc::k_moe_tc<3>};
    for (const void *k : ts) {
        cudaError_t e2 =
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, wf::mtc::SMEM);
        if (e2 != cudaSuccess) return cuda_fail(e2, "cudaFuncSetAttribute(moe tc)");
    }
    cudaError_t e = cudaFuncSetAttribute((const void *)wf::tc::k_dense_tc,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, wf::tc::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc)");
    e = cudaFuncSetAttribute((const void *)wf::tc::k_dense_tc_f32, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             wf::tc::F32_SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc f32)");
    e = cudaFuncSetAttribute((const void *)wf::fus::k_moe_fused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             wf::fus::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fused)");
    d.attr_done = true;
    return WF_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Tensor map of a [rows, K] weight matrix (FP4 packed or FP8), box 128 K x 128 rows,
// 128-byte swizzle; FP4 is unpacked to one byte per element in shared memory.
int weight_tensor_map(CUtensorMap *m, const void *base, bool fp4, uint64_t rows, uint64_t K,
                      uint32_t box_rows = 128) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(WF_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {fp4 ? K / 2 : K};
    const cuuint32_t box[2] = {128, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                     const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WF_E_SHAPE, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return WF_OK;
}

// Encoded tensor maps of the expert weights, cached by (pointer, shape):
// weights stay in place between calls, and encoding costs host time.
struct MapKey {
    const void *base;
    int dtype, rank;
    uint64_t dims[3], strides[2];
    uint32_t box[3];
    bool operator<(const MapKey &o) const { return memcmp(this, &o, sizeof(MapKey)) < 0; }
};
std::mutex g_map_mu;
std::map<MapKey, CUtensorMap> g_maps;

int cached_map(CUtensorMap *out, bool fp4, int rank, const void *base, const uint64_t *dims,
               const uint64_t *strides, const uint32_t *box) {
    MapKey k;
    memset(&k, 0, sizeof(k));
    k.base = base; k.dtype = fp4; k.rank = rank;
    for (int i = 0; i < rank; ++i) { k.dims[i] = dims[i]; k.box[i] = box[i]; }
    for (int i = 0; i + 1 < rank; ++i) k.strides[i] = strides[i];
    std::lock_guard<std::mutex> lock(g_map_mu);
    auto f = g_maps.find(k);
    if (f != g_maps.end()) { *out = f->second; return WF_OK; }
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(WF_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t d[3], st[2];
    cuuint32_t b[3], es[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) { d[i] = dims[i]; b[i] = box[i]; }
    for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
    CUresult r = enc(out, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, rank,
                     const_cast<void *>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WF_E_SHAPE, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps[k] = *out;
    return WF_OK;
}

// Bound of the kernels' waits on another role's progress; wf_set_wait_limit lowers it.
std::atomic<long long> g_wait_limit{wf::kWaitLimitCycles};

// Kernels this library has launched (or recorded into a stream capture) in this process.
std::atomic<unsigned long long> g_launches{0};
inline void counted(int n = 1) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

bool tc_disabled() {
    const char *v = getenv("WF_DISABLE_TC");
    return v && v[0] && v[0] != '0';
}

// WF_FUSED=1 runs the whole layer as the single fused launch (wf_moe_fused.cuh)
// instead of three launches (router, w1/w3, w2); expert parallelism over peer
// memory always uses the fused launch.
bool fused_requested() {
    const char *v = getenv("WF_FUSED");
    return v && v[0] && v[0] != '0';
}

// smem row stride: row bytes rounded up to 128, plus 16 (FP4: a warp reads one
// 4-byte word from each of 8 rows x 4 lanes) or 32 (FP8: 8 bytes from 8 rows x
// 4 lanes, two half-warp phases), so every access pattern is bank-conflict free
int stride_fp4(int K) { return ((K / 2 + 127) / 128) * 128 + 16; }
int stride_fp8(int K) { return ((K + 127) / 128) * 128 + 32; }

int rows_fit(int stride) {
    int r = wf::SLOT_W / stride;
    return r > wf::MAXR ? wf::MAXR : r;
}

// Grid bound of the tcgen05 expert phases (two stream-K partial slots per CTA).
constexpr int TC_MAX_GRID = 256;

struct WsLayout {
    size_t logits, hdr, act_expert, act_off, act_it2, act_it3, pair_tok, pair_w, tok_np,
        tok_pairs, ridx, rw, h, hs, o, os, cnt_router, cnt_rb, err, total;
    // tcgen05 expert phases: counters (zeroed region) and buffers after `total`
    size_t cnt_tc, xq, xs, hq, hqs, sq, sqs, part, total_tc;
    // the fused single-launch layer (wf_moe_fused.cuh): grid-barrier counter,
    // h-ready counters, per-class arrival counters, per-class partial slots
    size_t fgbar, fhcnt, fcnt, fpart, total_fused;
};

// Upper bound of the 16-token groups of one forward (shared + routed).
size_t tc_max_groups(const wf_moe_config *c) {
    const size_t T = c->max_tokens, K = c->topk, El = c->n_local_experts;
    return (T + 15) / 16 + std::min(El, T * K) + (T * K + 15) / 16;
}

// Upper bound of the items of one tcgen05 expert phase.
size_t tc_max_items(const wf_moe_config *c) {
    const size_t nblk = std::max((size_t)c->inter_dim / 128, (size_t)c->dim / 256);
    return tc_max_groups(c) * std::max<size_t>(nblk, 1);
}

// tc_counters = false: the layout of the allocation-free forward, which never runs
// the tcgen05 phases and so leaves out their per-item counters.
WsLayout ws_layout(const wf_moe_config *c, bool tc_counters = true) {
    WsLayout L{};
    size_t off = 0;
    const size_t T = c->max_tokens, K = c->topk, E = c->n_experts, El = c->n_local_experts;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align256(bytes);
        return o;
    };
    L.err = take(16);
    L.cnt_router = take(16);
    L.cnt_rb = take((size_t)(c->dim / 8 + 1) * 4);
    L.cnt_tc = take(tc_counters ? tc_max_items(c) * 4 : 0);
    L.hdr = take(wf::H_SIZE * 4);
    L.logits = take(T * E * 4);
    L.act_expert = take((El + 1) * 4);
    L.act_off = take((El + 1) * 4);
    L.act_it2 = take((El + 1) * 4);
    L.act_it3 = take((El + 1) * 4);
    L.pair_tok = take(T * K * 4);
    L.pair_w = take(T * K * 4);
    L.tok_np = take(T * 4);
    L.tok_pairs = take(T * K * 4);
    L.ridx = take(T * K * 4);
    L.rw = take(T * K * 4);
    L.h = take(T * K * c->inter_dim * 2);
    L.hs = take(T * c->inter_dim * 2);
    L.o = take(T * K * c->dim * 2);
    L.os = take(T * c->dim * 2);
    L.total = off;
    const size_t D = c->dim, I = c->inter_dim;
    L.xq = take(T * D);
    L.xs = take(T * D / 128);
    L.hq = take(T * K * I);
    L.hqs = take(T * K * I / 128);
    L.sq = take(T * I);
    L.sqs = take(T * I / 128);
    L.part = take((size_t)TC_MAX_GRID * 2 * (2 * 128 * wf::mtc::NT) * 4);
    L.total_tc = off;
    L.fgbar = take(16);
    L.fhcnt = take(tc_max_groups(c) * 4);
    L.fcnt = take(4 * tc_max_items(c) * 4);
    L.fpart = take((size_t)TC_MAX_GRID * 8 * (2 * 128 * wf::mtc::NT) * 4);
    L.total_fused = off;
    return L;
}

int check_cfg(const wf_moe_config *c) {
    if (!c) return fail(WF_E_ARG, "null config");
    const int D = c->dim, I = c->inter_dim;
    if (D <= 0 || I <= 0 || D % 128 || I % 128 || D > wf::KMAX || I > wf::KMAX)
        return fail(WF_E_SHAPE, "dim and inter_dim must be positive multiples of 128, at most 4096");
    if (c->n_experts <= 0 || c->n_experts > wf::MAX_E)
        return fail(WF_E_SHAPE, "n_experts must be in 1..512");
    if (c->n_local_experts <= 0 || c->expert_offset < 0 ||
        c->expert_offset + c->n_local_experts > c->n_experts)
        return fail(WF_E_SHAPE, "local expert range outside [0, n_experts)");
    if (c->topk <= 0 || c->topk > wf::MAX_K || c->topk > c->n_experts)
        return fail(WF_E_SHAPE, "topk must be in 1..min(8, n_experts)");
    if (c->score_func < 0 || c->score_func > 2) return fail(WF_E_DTYPE, "bad score_func");
    if (c->max_tokens <= 0 || c->max_tokens > wf::MAX_T)
        return fail(WF_E_SHAPE, "max_tokens must be in 1..256");
    if (c->hash_layer && c->vocab <= 0) return fail(WF_E_SHAPE, "hash layer needs vocab > 0");
    return WF_OK;
}

wf::Geo make_geo(int D, int I) {
    wf::Geo g;
    g.st_w13 = stride_fp4(D);
    g.st_w2 = stride_fp4(I);
    g.st_s13 = stride_fp8(D);
    g.st_s2 = stride_fp8(I);
    auto pick_h = [&](int stride) {  // h-rows per SwiGLU item: 2*nh rows, nh | I
        int r = rows_fit(stride) / 2;
        int nh = r >= 16 ? 16 : r >= 8 ? 8 : 4;
        while (I % nh) nh /= 2;
        return nh;
    };
    auto pick_r = [&](int stride) {  // rows per plain item: 32, 16 or 8, divides D
        const int fit = rows_fit(stride);
        int r = fit >= 32 ? 32 : fit >= 16 ? 16 : 8;
        while (D % r) r /= 2;
        return r;
    };
    g.nh13 = pick_h(g.st_w13);
    g.nhs13 = pick_h(g.st_s13);
    g.r2 = pick_r(g.st_w2);
    g.rs2 = pick_r(g.st_s2);
    return g;
}

// Expert phases on tcgen05: needs power-of-two (e8m0) activation and shared
// scales, 256-row output blocks, the tcgen05 workspace, aligned weight banks.
int fill_tc(const wf_moe_config *c, const wf_moe_weights *w, const WsLayout &L, uint8_t *b,
            size_t ws_bytes, wf::MoeArgs &a, wf::mtc::TcArgs *t, wf::fus::FArgs *f = nullptr,
            bool force_fused = false) {
    a.tc = 0;
    if (f) f->gbar = nullptr;
    if (!t || tc_disabled()) return WF_OK;
    const int D = c->dim, I = c->inter_dim, El = c->n_local_experts;
    if (!c->ue8m0 || w->shared_scale_kind == WF_SCALE_F32 || D % 256 || ws_bytes < L.total_tc) return WF_OK;
    auto al = [](const void *p) { return ((uintptr_t)p & 255) == 0; };
    if (!al(w->w13) || !al(w->w2) || !al(w->shared_w13) || !al(w->shared_w2)) return WF_OK;
    memset(t, 0, sizeof(*t));
    int rc;
    {
        const uint64_t dims[3] = {(uint64_t)D, (uint64_t)I, 2ull * El};
        const uint64_t st[2] = {(uint64_t)D / 2, (uint64_t)I * D / 2};
        const uint32_t box[3] = {128, 128, 2};
        if ((rc = cached_map(&t->m_r13, true, 3, w->w13, dims, st, box))) return rc;
    }
    {
        const uint64_t dims[3] = {(uint64_t)D, (uint64_t)I, 2};
        const uint64_t st[2] = {(uint64_t)D, (uint64_t)I * D};
        const uint32_t box[3] = {128, 128, 2};
        if ((rc = cached_map(&t->m_s13, false, 3, w->shared_w13, dims, st, box))) return rc;
    }
    {
        const uint64_t dims[2] = {(uint64_t)I, (uint64_t)El * D};
        const uint64_t st[1] = {(uint64_t)I / 2};
        const uint32_t box[2] = {128, 256};
        if ((rc = cached_map(&t->m_r2, true, 2, w->w2, dims, st, box))) return rc;
    }
    {
        const uint64_t dims[2] = {(uint64_t)I, (uint64_t)D};
        const uint64_t st[1] = {(uint64_t)I};
        const uint32_t box[2] = {128, 256};
        if ((rc = cached_map(&t->m_s2, false, 2, w->shared_w2, dims, st, box))) return rc;
    }
    a.tc = 1;
    a.xq = b + L.xq; a.xs = b + L.xs;
    t->xq = a.xq; t->xs = a.xs;
    t->hq = b + L.hq; t->hqs = b + L.hqs;
    t->sq = b + L.sq; t->sqs = b + L.sqs;
    t->part = (float *)(b + L.part);
    t->cnt = (unsigned *)(b + L.cnt_tc);
    if (f && (force_fused || fused_requested()) && ws_bytes >= L.total_fused) {
        f->gbar = (unsigned long long *)(b + L.fgbar);
        f->hcnt = (unsigned *)(b + L.fhcnt);
        f->cnt = (unsigned *)(b + L.fcnt);
        f->part = (float *)(b + L.fpart);
        f->max_items = (int)tc_max_items(c);
    }
    // items of 128 h-rows (w1/w3) and 256 output rows (w2) in the dispatch tables
    a.g.nh13 = 128;
    a.g.r2 = 256;
    return WF_OK;
}

int fill_args(const wf_moe_config *c, const wf_moe_weights *w, const void *x,
              const int64_t *ids, int T, void *ws, size_t ws_bytes, wf::MoeArgs &a,
              wf::mtc::TcArgs *t = nullptr, bool routing_given = false, bool tc_counters = true,
              wf::fus::FArgs *f = nullptr, bool force_fused = false) {
    int rc = check_cfg(c);
    if (rc) return rc;
    if (!w || !x || !ws) return fail(WF_E_ARG, "null weights, input or workspace");
    if (T <= 0 || T > c->max_tokens) return fail(WF_E_SHAPE, "T outside 1..max_tokens");
    const WsLayout L = ws_layout(c, tc_counters);
    if (ws_bytes < L.total) return fail(WF_E_ARG, "workspace too small");
    if (!w->gate_w) return fail(WF_E_ARG, "null gate weight");
    if (c->hash_layer && !routing_given && (!w->tid2eid || !ids))
        return fail(WF_E_ARG, "hash layer needs tid2eid and input_ids");
    memset(&a, 0, sizeof(a));
    a.sh0 = 0; a.shT = T; a.sh_add = 1;  // the shared expert on every row, added by the combine
    a.T = T; a.D = c->dim; a.I = c->inter_dim; a.E = c->n_experts; a.El = c->n_local_experts;
    a.e0 = c->expert_offset; a.topk = c->topk; a.score_func = c->score_func;
    a.hash = c->hash_layer; a.ue8m0 = c->ue8m0; a.vocab = c->vocab;
    a.route_scale = c->route_scale; a.swiglu_limit = c->swiglu_limit;
    a.x = (const __nv_bfloat16 *)x; a.ids = (const long long *)ids;
    a.gate_w = (const __nv_bfloat16 *)w->gate_w; a.gate_b = c->hash_layer ? nullptr : w->gate_bias;
    a.tid2eid = w->tid2eid;
    a.w13 = w->w13; a.w13_s = w->w13_s; a.w2 = w->w2; a.w2_s = w->w2_s;
    a.sw13 = w->shared_w13; a.sw2 = w->shared_w2; a.ss13 = w->shared_s13; a.ss2 = w->shared_s2;
    a.shared_f32 = w->shared_scale_kind == WF_SCALE_F32;
    uint8_t *b = (uint8_t *)ws;
    a.logits = (float *)(b + L.logits);
    a.hdr = (int *)(b + L.hdr);
    a.act_expert = (int *)(b + L.act_expert);
    a.act_off = (int *)(b + L.act_off);
    a.act_it2 = (int *)(b + L.act_it2);
    a.act_it3 = (int *)(b + L.act_it3);
    a.pair_tok = (int *)(b + L.pair_tok);
    a.pair_w = (float *)(b + L.pair_w);
    a.tok_np = (int *)(b + L.tok_np);
    a.tok_pairs = (int *)(b + L.tok_pairs);
    a.ridx = (int *)(b + L.ridx);
    a.rw = (float *)(b + L.rw);
    a.h = (__nv_bfloat16 *)(b + L.h);
    a.hs = (__nv_bfloat16 *)(b + L.hs);
    a.o = (__nv_bfloat16 *)(b + L.o);
    a.os = (__nv_bfloat16 *)(b + L.os);
    a.cnt_router = (unsigned *)(b + L.cnt_router);
    a.cnt_rb = (unsigned *)(b + L.cnt_rb);
    a.err = (int *)(b + L.err);
    a.g = make_geo(a.D, a.I);
    return fill_tc(c, w, L, b, ws_bytes, a, t, f, force_fused);
}

}  // namespace

extern "C" {

const char *wf_last_error(void) { return g_err.c_str(); }

int wf_device_sm_count(void) { return sm_count(); }

size_t wf_moe_workspace_bytes(const wf_moe_config *cfg) {
    if (check_cfg(cfg)) return 0;
    return ws_layout(cfg).total_fused;
}

static int launch_moe(wf::MoeArgs &a, bool route_only, cudaStream_t st,
                      void *const *ev = nullptr, const wf::mtc::TcArgs *t = nullptr,
                      const wf::fus::FArgs *f = nullptr) {
    int rc = ensure_attrs();
    if (rc) return rc;
    int G = sm_count();
    if (G <= 0) return fail(WF_E_CUDA, "no CUDA device");
    a.route_only = route_only;
    a.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
    if (a.tc && !t) return fail(WF_E_ARG, "tcgen05 phases without their arguments");
    // Programmatic dependent launch: a kernel may begin launching while the one
    // before it drains; each kernel waits (griddepcontrol.wait) before reading
    // anything an earlier kernel wrote.  Event records break the overlap on
    // purpose, so the timed variant launches without it.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ev ? 0 : 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(G);
    lc.blockDim = dim3(wf::NTHR);
    lc.dynamicSmemBytes = wf::SMEM_BYTES;
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 1;
    cudaLaunchConfig_t lt = lc;
    lt.gridDim = dim3(std::min(G, TC_MAX_GRID));
    lt.blockDim = dim3(wf::mtc::THREADS);
    lt.dynamicSmemBytes = wf::mtc::SMEM;
    cudaError_t e = cudaSuccess;
    auto rec = [&](int i) {
        if (ev && e == cudaSuccess)
            e = cudaEventRecordWithFlags((cudaEvent_t)ev[i], st, cudaEventRecordDefault);
    };
    if (!route_only && a.tc && f && f->gbar) {
        // the whole layer in one launch; the timing events bracket it (0 -> 1),
        // and events 2 and 3 mark the same end point
        cudaLaunchConfig_t lf = lt;
        lf.dynamicSmemBytes = wf::fus::SMEM;
        rec(0);
        if (e == cudaSuccess && (e = cudaLaunchKernelEx(&lf, wf::fus::k_moe_fused, a, *t, *f)) == cudaSuccess)
            counted();
        rec(1);
        rec(2);
        rec(3);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "fused MoE kernel launch");
        return WF_OK;
    }
    rec(0);
    if (e == cudaSuccess && (e = cudaLaunchKernelEx(&lc, wf::k_moe_up, a)) == cudaSuccess) counted();
    rec(1);
    if (!route_only) {
        if (a.tc) {
            if (e == cudaSuccess && (e = cudaLaunchKernelEx(&lt, wf::mtc::k_moe_tc<2>, a, *t)) == cudaSuccess) counted();
            rec(2);
            if (e == cudaSuccess && (e = cudaLaunchKernelEx(&lt, wf::mtc::k_moe_tc<3>, a, *t)) == cudaSuccess) counted();
            rec(3);
        } else {
            if (e == cudaSuccess && (e = cudaLaunchKernelEx(&lc, wf::k_moe_mid, a)) == cudaSuccess) counted();
            rec(2);
            if (e == cudaSuccess && (e = cudaLaunchKernelEx(&lc, wf::k_moe_down, a)) == cudaSuccess) counted();
            rec(3);
        }
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "MoE kernel launch");
    return WF_OK;
}

static int check_expert_ptrs(const wf_moe_weights *w) {
    if (!w) return fail(WF_E_ARG, "null weights");
    if (!w->w13 || !w->w13_s || !w->w2 || !w->w2_s || !w->shared_w13 || !w->shared_s13 ||
        !w->shared_w2 || !w->shared_s2)
        return fail(WF_E_ARG, "null expert weight pointer");
    return WF_OK;
}

int wf_moe_forward(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                   const int64_t *input_ids, int32_t T, void *y, float *y_partial,
                   float *out_weights, int64_t *out_indices, void *workspace,
                   size_t workspace_bytes, void *stream) {
    int rc = check_expert_ptrs(w);
    if (rc) return rc;
    wf::MoeArgs a;
    wf::mtc::TcArgs t;
    wf::fus::FArgs f;
    rc = fill_args(cfg, w, x, input_ids, T, workspace, workspace_bytes, a, &t, false, true, &f);
    if (rc) return rc;
    if (!y && !y_partial) return fail(WF_E_ARG, "need y or y_partial");
    a.y = (__nv_bfloat16 *)y; a.y_partial = y_partial; a.partial = y_partial != nullptr;
    a.sh_add = !a.partial;  // a partial forward leaves the shared rows to wf_moe_finish
    a.out_w = out_weights; a.out_idx = (long long *)out_indices;
    return launch_moe(a, false, (cudaStream_t)stream, nullptr, &t, &f);
}

int wf_moe_forward_timed(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                         const int64_t *input_ids, int32_t T, void *y, float *y_partial,
                         float *out_weights, int64_t *out_indices, void *workspace,
                         size_t workspace_bytes, void *stream, void *const *events) {
    if (!events) return fail(WF_E_ARG, "null events");
    for (int i = 0; i < 4; ++i)
        if (!events[i]) return fail(WF_E_ARG, "null event");
    int rc = check_expert_ptrs(w);
    if (rc) return rc;
    wf::MoeArgs a;
    wf::mtc::TcArgs t;
    wf::fus::FArgs f;
    rc = fill_args(cfg, w, x, input_ids, T, workspace, workspace_bytes, a, &t, false, true, &f);
    if (rc) return rc;
    if (!y && !y_partial) return fail(WF_E_ARG, "need y or y_partial");
    a.y = (__nv_bfloat16 *)y; a.y_partial = y_partial; a.partial = y_partial != nullptr;
    a.sh_add = !a.partial;  // a partial forward leaves the shared rows to wf_moe_finish
    a.out_w = out_weights; a.out_idx = (long long *)out_indices;
    return launch_moe(a, false, (cudaStream_t)stream, events, &t, &f);
}

int wf_moe_forward_ep(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x, int32_t T,
                      const float *in_weights, const int64_t *in_indices, int32_t shared_row0,
                      int32_t shared_rows, float *y_partial, void *workspace, size_t workspace_bytes,
                      void *stream) {
    int rc = check_expert_ptrs(w);
    if (rc) return rc;
    if (!in_weights || !in_indices || !y_partial) return fail(WF_E_ARG, "null routing or output");
    if (shared_row0 < 0 || shared_rows < 0 || (int64_t)shared_row0 + shared_rows > T)
        return fail(WF_E_SHAPE, "shared rows outside 0..T");
    wf::MoeArgs a;
    wf::mtc::TcArgs t;
    wf::fus::FArgs f;
    rc = fill_args(cfg, w, x, nullptr, T, workspace, workspace_bytes, a, &t, true, true, &f);
    if (rc) return rc;
    a.given = 1;
    a.in_w = in_weights; a.in_idx = (const long long *)in_indices;
    a.sh0 = shared_row0; a.shT = shared_rows; a.sh_add = 1;
    a.y = nullptr; a.y_partial = y_partial; a.partial = 1;
    a.out_w = nullptr; a.out_idx = nullptr;
    return launch_moe(a, false, (cudaStream_t)stream, nullptr, &t, &f);
}

int wf_moe_sum_ranks(const float *parts, int32_t P, int64_t n, void *y, void *stream) {
    if (!parts || !y) return fail(WF_E_ARG, "null pointer");
    if (P <= 0 || P > 1024) return fail(WF_E_SHAPE, "P outside 1..1024");
    if (n <= 0 || n % 4 || n > (int64_t)1 << 30) return fail(WF_E_SHAPE, "n must be a positive multiple of 4 up to 2^30");
    if ((uintptr_t)parts % 16 || (uintptr_t)y % 8) return fail(WF_E_ARG, "parts must be 16-byte and y 8-byte aligned");
    const int64_t n4 = n / 4, blocks = (n4 + 255) / 256;
    wf::k_sum_ranks<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, (cudaStream_t)stream>>>(
        (const float4 *)parts, P, n4, (uint2 *)y); counted();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "sum_ranks launch");
}

int wf_moe_to_bf16(const float *src, int64_t n, void *dst, void *stream) {
    if (!src || !dst) return fail(WF_E_ARG, "null pointer");
    if (n <= 0 || n > (int64_t)1 << 30) return fail(WF_E_SHAPE, "n outside 1..2^30");
    const int64_t blocks = (n + 255) / 256;
    wf::k_to_bf16<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, (cudaStream_t)stream>>>(
        src, (__nv_bfloat16 *)dst, (int)n); counted();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "to_bf16 launch");
}

int wf_moe_route(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                 const int64_t *input_ids, int32_t T, float *out_weights, int64_t *out_indices,
                 void *workspace, size_t workspace_bytes, void *stream) {
    wf::MoeArgs a;
    int rc = fill_args(cfg, w, x, input_ids, T, workspace, workspace_bytes, a);
    if (rc) return rc;
    if (!out_weights || !out_indices) return fail(WF_E_ARG, "null router outputs");
    a.out_w = out_weights; a.out_idx = (long long *)out_indices;
    return launch_moe(a, true, (cudaStream_t)stream);
}

int wf_moe_finish(const wf_moe_config *cfg, const float *yp, int32_t T, int32_t row0, void *y,
                  const void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (!yp || !y || !workspace) return fail(WF_E_ARG, "null pointer");
    const WsLayout L = ws_layout(cfg);
    if (workspace_bytes < L.total) return fail(WF_E_ARG, "workspace too small");
    if (T <= 0 || row0 < 0 || row0 + T > cfg->max_tokens)
        return fail(WF_E_SHAPE, "rows row0..row0+T outside 0..max_tokens");
    const int n = T * cfg->dim;
    const __nv_bfloat16 *os =
        (const __nv_bfloat16 *)((const uint8_t *)workspace + L.os) + (size_t)row0 * cfg->dim;
    wf::k_moe_finish<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(yp, os, (__nv_bfloat16 *)y, n); counted();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "finish launch");
}

// ---------------------------------------------------------------------------
// Expert parallelism over peer memory.  Every rank holds one buffer of the same
// layout; the ranks map each other's buffers (CUDA IPC) and the fused kernel
// writes tokens, routing and partial output rows straight into them.
// ---------------------------------------------------------------------------
struct EpLayout {
    size_t flags, xq, xs, ridx, rw, yrecv, total;
};

static EpLayout ep_layout(const wf_moe_config *c, int world) {
    EpLayout L{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align256(bytes);
        return o;
    };
    const size_t Tg = (size_t)c->max_tokens, D = c->dim, K = c->topk;
    const size_t Tr = Tg / (size_t)std::max(world, 1);
    L.flags = take(wf::EP_FLAG_WORDS * 4);
    L.xq = take(Tg * D);
    L.xs = take(Tg * D / 128);
    L.ridx = take(Tg * K * 4);
    L.rw = take(Tg * K * 4);
    L.yrecv = take((size_t)world * Tr * D * 4);
    L.total = off;
    return L;
}

size_t wf_ep_buffer_bytes(const wf_moe_config *cfg, int32_t world) {
    if (check_cfg(cfg)) return 0;
    if (world < 1 || world > wf::EP_MAX_RANKS) return (size_t)fail(WF_E_SHAPE, "world outside 1..8"), 0;
    return ep_layout(cfg, world).total;
}

int wf_ep_alloc(size_t bytes, void **buf) {
    if (!buf || !bytes) return fail(WF_E_ARG, "null output or zero size");
    cudaError_t e = cudaMalloc(buf, bytes);
    if (e == cudaSuccess) e = cudaMemset(*buf, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "expert-parallel buffer");
}

int wf_ep_free(void *buf) {
    cudaError_t e = cudaFree(buf);
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "cudaFree(expert-parallel buffer)");
}

int wf_ipc_get_handle(const void *buf, void *handle) {
    if (!buf || !handle) return fail(WF_E_ARG, "null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(buf));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == WF_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return WF_OK;
}

int wf_ipc_open_handle(const void *handle, void **buf) {
    if (!buf || !handle) return fail(WF_E_ARG, "null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int wf_ipc_close_handle(void *buf) {
    cudaError_t e = cudaIpcCloseMemHandle(buf);
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int wf_moe_forward_ep_p2p(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                          const int64_t *input_ids, int32_t T, int32_t rank, int32_t world,
                          void *const *bufs, void *y, float *out_weights, int64_t *out_indices,
                          void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_expert_ptrs(w);
    if (rc) return rc;
    if (!bufs || !y) return fail(WF_E_ARG, "null buffers or output");
    if (world < 1 || world > wf::EP_MAX_RANKS || rank < 0 || rank >= world)
        return fail(WF_E_SHAPE, "rank / world outside 0..world-1 / 1..8");
    if (T <= 0 || (int64_t)T * world > cfg->max_tokens)
        return fail(WF_E_SHAPE, "world * T exceeds max_tokens (the gathered batch's capacity)");
    for (int p = 0; p < world; ++p)
        if (!bufs[p]) return fail(WF_E_ARG, "null peer buffer");
    wf::MoeArgs a;
    wf::mtc::TcArgs t;
    wf::fus::FArgs f;
    rc = fill_args(cfg, w, x, input_ids, T * world, workspace, workspace_bytes, a, &t, false, true, &f, true);
    if (rc) return rc;
    if (!a.tc || !f.gbar)
        return fail(WF_E_ARG, "expert parallelism over peer memory needs the fused tcgen05 engine "
                              "(e8m0 scales, the full workspace, WF_DISABLE_TC unset)");
    const EpLayout E = ep_layout(cfg, world);
    a.ep = 1; a.ep_rank = rank; a.ep_world = world; a.Tr = T;
    for (int p = 0; p < world; ++p) {
        uint8_t *b = (uint8_t *)bufs[p];
        a.ep_xq[p] = b + E.xq; a.ep_xs[p] = b + E.xs;
        a.ep_ridx[p] = (int *)(b + E.ridx); a.ep_rw[p] = (float *)(b + E.rw);
        a.ep_yrecv[p] = (float *)(b + E.yrecv); a.ep_flags[p] = (unsigned *)(b + E.flags);
    }
    uint8_t *mine = (uint8_t *)bufs[rank];
    a.xq = mine + E.xq;  // the gathered batch lives in this rank's buffer
    a.xs = mine + E.xs;
    t.xq = a.xq;
    t.xs = a.xs;
    a.ridx = (int *)(mine + E.ridx);
    a.rw = (float *)(mine + E.rw);
    a.ep_done = a.cnt_router;  // a workspace counter no other path of the fused engine uses
    a.sh0 = rank * T; a.shT = T; a.sh_add = 1;  // the shared expert on this rank's tokens
    a.y = nullptr; a.y_partial = nullptr; a.partial = 1;
    a.out_w = out_weights; a.out_idx = (long long *)out_indices;
    rc = launch_moe(a, false, (cudaStream_t)stream, nullptr, &t, &f);
    if (rc) return rc;
    const int64_t n = (int64_t)T * cfg->dim;
    const int blocks = (int)std::min<int64_t>(1024, (n + 255) / 256);
    wf::fus::k_ep_finish<<<blocks, 256, 0, (cudaStream_t)stream>>>(
        (unsigned *)(mine + E.flags), (const float *)(mine + E.yrecv), world, T, cfg->dim,
        (__nv_bfloat16 *)y, a.err, a.wait_limit); counted();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "expert-parallel finish launch");
}

// ---------------------------------------------------------------------------
// Allocation-free forward.  Some callers cannot give the layer a workspace:
// their device memory is owned by another allocator that hands out nothing
// at call time, or they may not call into the CUDA allocator on a
// latency-critical path (cudaMalloc can synchronize the device).  For them
// the scratch lives in this library's own module-scope device array, created
// when the module loads on a device and held until the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_noalloc_scratch[WF_NOALLOC_SCRATCH_BYTES];

// cuCtxGetCurrent through the runtime's driver entry point (no libcuda link).
typedef CUresult (*CtxGetCurrentFn)(CUcontext *);

static CtxGetCurrentFn ctx_get_current_fn() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    return fn;
}

static std::mutex g_noalloc_mu;
static std::map<std::pair<int, CUcontext>, void *> g_noalloc_ptr;

// Device address of g_noalloc_scratch for the current device and context,
// looked up once per (device, context) with that device current.  In host code
// the array's name is only a stand-in; a kernel must get this address.
static int noalloc_scratch(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    CtxGetCurrentFn get = ctx_get_current_fn();
    if (!get) return fail(WF_E_CUDA, "cuCtxGetCurrent unavailable");
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS) return fail(WF_E_CUDA, "cuCtxGetCurrent failed");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (ctx) {
        auto f = g_noalloc_ptr.find(std::make_pair(dev, ctx));
        if (f != g_noalloc_ptr.end()) {
            *out = f->second;
            return WF_OK;
        }
    }
    // first call in this context: the lookup also makes the device's primary
    // context current when the calling thread had none
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    if (get(&ctx) != CUDA_SUCCESS || !ctx) return fail(WF_E_CUDA, "no current CUDA context");
    g_noalloc_ptr[std::make_pair(dev, ctx)] = p;
    *out = p;
    return WF_OK;
}

int wf_moe_forward_noalloc(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                           const int64_t *input_ids, int32_t T, void *y, float *out_weights,
                           int64_t *out_indices, void *stream) {
    if (!cfg) return fail(WF_E_ARG, "null config");
    if (T <= 0) return fail(WF_E_SHAPE, "T must be positive");
    wf_moe_config c = *cfg;
    c.max_tokens = T;  // size the scratch for this call only
    int rc = check_cfg(&c);
    if (rc) return rc;
    const WsLayout L = ws_layout(&c, false);
    if (L.total > WF_NOALLOC_SCRATCH_BYTES)
        return fail(WF_E_SHAPE, "T too large for the static scratch of wf_moe_forward_noalloc (" +
                                    std::to_string(L.total) + " bytes needed, " +
                                    std::to_string((size_t)WF_NOALLOC_SCRATCH_BYTES) + " available)");
    rc = check_expert_ptrs(w);
    if (rc) return rc;
    if (!y) return fail(WF_E_ARG, "null output");
    void *scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    wf::MoeArgs a;
    rc = fill_args(&c, w, x, input_ids, T, scratch, WF_NOALLOC_SCRATCH_BYTES, a, nullptr, false, false);
    if (rc) return rc;
    // The completion counters must start at zero (a call that timed out can leave
    // them set); the rest is fully written before it is read.  The error word at
    // the start of the array is left alone: it collects every call's flags until
    // wf_moe_read_error_noalloc reads and clears it.
    cudaError_t e = cudaMemsetAsync((uint8_t *)scratch + L.cnt_router, 0, L.logits - L.cnt_router,
                                    (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(scratch counters)");
    a.y = (__nv_bfloat16 *)y; a.y_partial = nullptr; a.partial = 0;
    a.out_w = out_weights; a.out_idx = (long long *)out_indices;
    return launch_moe(a, false, (cudaStream_t)stream);
}

// Reads (synchronizing `stream`) and clears the error word of the static scratch.
static int read_error_word(void *word, cudaStream_t st) {
    int host = 0;
    cudaError_t e = cudaMemcpyAsync(&host, word, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "read error word");
    if (host) {
        // read-and-clear: the next read reports only what later calls set
        e = cudaMemsetAsync(word, 0, 4, st);
        if (e != cudaSuccess) return cuda_fail(e, "clear error word");
    }
    if (host & wf::kErrTimeout) return fail(WF_E_TIMEOUT, "a device wait timed out");
    if (host & wf::kErrExpertId) return fail(WF_E_EXPERT_ID, "token or expert id out of range");
    return WF_OK;
}

int wf_moe_read_error_noalloc(void *stream) {
    void *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    return read_error_word(scratch, (cudaStream_t)stream);
}

uint64_t wf_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int wf_set_wait_limit(int64_t cycles) {
    g_wait_limit.store(cycles > 0 ? (long long)cycles : wf::kWaitLimitCycles, std::memory_order_relaxed);
    return WF_OK;
}

int wf_moe_read_error(const void *workspace, size_t workspace_bytes, void *stream) {
    if (!workspace || workspace_bytes < 16) return fail(WF_E_ARG, "null workspace");
    return read_error_word(const_cast<void *>(workspace), (cudaStream_t)stream);
}

int wf_act_quant(const void *x, int64_t M, int64_t K, int32_t block, int32_t ue8m0, void *q,
                 void *s, int32_t scale_kind, void *stream) {
    if (!x || !q || !s) return fail(WF_E_ARG, "null pointer");
    if (M <= 0 || K <= 0 || block <= 0 || K % block) return fail(WF_E_SHAPE, "K must be a multiple of block");
    if (scale_kind != WF_SCALE_F32 && scale_kind != WF_SCALE_E8M0) return fail(WF_E_DTYPE, "bad scale kind");
    if (scale_kind == WF_SCALE_E8M0 && !ue8m0) return fail(WF_E_DTYPE, "e8m0 scales need ue8m0 rounding");
    const long long warps = M * (K / block);
    const long long blocks = (warps * 32 + 255) / 256;
    wf::k_act_quant<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)x, M, K, block, ue8m0, (uint8_t *)q, s, scale_kind == WF_SCALE_F32); counted();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "act_quant launch");
}

int wf_fp4_act_quant(const void *x, int64_t M, int64_t K, void *q, void *s, void *stream) {
    if (!x || !q || !s) return fail(WF_E_ARG, "null pointer");
    if (M <= 0 || K <= 0 || K % 32) return fail(WF_E_SHAPE, "K must be a multiple of 32");
    const long long n = M * (K / 32);
    wf::k_fp4_act_quant<<<(unsigned)((n + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)x, M, K, (uint8_t *)q, (uint8_t *)s); counted();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "fp4_act_quant launch");
}

static int gemm_chunks(int64_t K) { return (int)((K + wf::KMAX - 1) / wf::KMAX); }

// K chunks of the tcgen05 dense path: at least enough to fill ~2 items per SM
// when there are few 128-row tiles, each chunk a multiple of 128 and <= 4096.
// K split of the tcgen05 dense GEMM: the number of chunks that minimizes an
// estimate of the kernel time.  Items (16 tokens x 128 rows x one K chunk) are
// dealt to the SMs in rounds; an item costs its K steps at the per-SM share of
// the streaming rate (5.5 TB/s over 148 SMs, ~37 GB/s; 16 KB of HBM per step
// for E4M3, 8 KB for E2M1) plus ~2 us of fixed work (B operand, scales,
// epilogue), and the split-K sum adds ~0.5 us per chunk.  A finer split only
// pays while it fills idle SMs.
static int tc_chunks(int64_t M, int64_t N, int64_t K, bool fp4) {
    const int64_t sms = std::max(1, sm_count());
    const int64_t items = ((M + 15) / 16) * (N / 128);
    const double step_us = (fp4 ? 8192.0 : 16384.0) / 37.0e3;
    int best = 0;
    double best_us = 1e30;
    for (int nkc = gemm_chunks(K); nkc <= 16; nkc *= 2) {
        if (K % (128 * nkc) || K / nkc > wf::tc::KC_MAX) continue;
        const int64_t rounds = (items * nkc + sms - 1) / sms;
        const double us = (double)rounds * ((double)(K / nkc / 128) * step_us + 2.0) + (nkc > 1 ? 0.5 * nkc : 0.0);
        if (us < best_us) { best_us = us; best = nkc; }
    }
    return best > 0 ? best : gemm_chunks(K);
}

static int gemm_rows(int wfmt, int64_t N, int64_t K) {
    const int nkc = gemm_chunks(K);
    const int Kc = (int)(K / nkc);
    const int fit = rows_fit(wfmt == wf::FMT_FP4 ? stride_fp4(Kc) : stride_fp8(Kc));
    return (fit >= 32 && N % 32 == 0) ? 32 : (fit >= 16 && N % 16 == 0) ? 16 : 8;
}

struct GemmWs {
    size_t cnt, part, total;
};

static GemmWs gemm_ws(int64_t M, int64_t N, int64_t K, int rows) {
    GemmWs w{};
    const int nkc = gemm_chunks(K);
    w.cnt = 256;
    if (nkc <= 1) { w.part = w.total = 256; return w; }
    // counters per (token group or slot, row block): M * N/rows bounds both cases
    const size_t groups = (size_t)M * (N / rows);
    w.part = w.cnt + align256(groups * 4);
    w.total = w.part + align256((size_t)nkc * M * N * 4);
    return w;
}

// tcgen05 dense path: counters per (token group, 128-row tile, lane quadrant) + partials
static GemmWs gemm_ws_tc(int64_t M, int64_t N, int64_t K, int nkc) {
    GemmWs w{};
    w.cnt = 256;
    if (nkc <= 1) { w.part = w.total = 256; return w; }
    w.part = w.cnt + align256((size_t)((M + 15) / 16) * (N / 128) * 4 * 4);
    w.total = w.part + align256((size_t)nkc * M * N * 4);
    return w;
}

size_t wf_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0 || N % 8) return 0;
    // sized for the finer of the FP8 / FP4 row blockings, and for the tcgen05 split-K
    const int rows = std::min(gemm_rows(wf::FMT_FP8, N, K), gemm_rows(wf::FMT_FP4, N, K));
    size_t need = gemm_ws(M, N, K, rows).total;
    if (N % 128 == 0 && K % 128 == 0)
        need = std::max({need, gemm_ws_tc(M, N, K, tc_chunks(M, N, K, false)).total,
                         gemm_ws_tc(M, N, K, tc_chunks(M, N, K, true)).total});
    return need;
}

// The split-K counters of a GEMM workspace return to zero at the end of every
// call (the last chunk of each tile resets its counter), but where the counter
// and partial regions lie depends on the shape, so a workspace is cleared when
// the shape it serves changes.  Skipping the clear otherwise keeps consecutive
// GEMMs of one shape adjacent on the stream, so programmatic dependent launch
// overlaps each one's set-up and weight stream with the previous one.
struct GemmShape {
    int64_t M, N, K;
    int fmt;
    bool operator==(const GemmShape &o) const { return M == o.M && N == o.N && K == o.K && fmt == o.fmt; }
};
static std::mutex g_gemm_shape_mu;
static std::map<const void *, GemmShape> g_gemm_shape;

static bool gemm_shape_changed(const void *ws, const GemmShape &sh) {
    std::lock_guard<std::mutex> lock(g_gemm_shape_mu);
    auto it = g_gemm_shape.find(ws);
    if (it != g_gemm_shape.end() && it->second == sh) return false;
    g_gemm_shape[ws] = sh;
    return true;
}

static int dense(int wfmt, const void *a, const void *a_s, int a_kind, const void *b,
                 const void *b_s, int b_kind, int64_t M, int64_t N, int64_t K, int64_t G,
                 void *out, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!a || !a_s || !b || !b_s || !out || !ws) return fail(WF_E_ARG, "null pointer");
    const int nkc = K > 0 ? gemm_chunks(K) : 0;
    if (M <= 0 || N <= 0 || K <= 0 || N % 8 || K % (128 * nkc))
        return fail(WF_E_SHAPE, "need N a multiple of 8 and K a multiple of 128 per 4096-wide chunk");
    if ((a_kind != WF_SCALE_F32 && a_kind != WF_SCALE_E8M0) ||
        (b_kind != WF_SCALE_F32 && b_kind != WF_SCALE_E8M0))
        return fail(WF_E_DTYPE, "bad scale kind");
    if (M > (1 << 24) || N > (1 << 26) || G > (1 << 16) || K > (1 << 20)) return fail(WF_E_SHAPE, "too large");
    const int rows = gemm_rows(wfmt, N, K);
    const GemmWs L = gemm_ws(G > 0 ? G : M, N, K, rows);
    if (ws_bytes < L.total) return fail(WF_E_ARG, "workspace too small (see wf_gemm_workspace_bytes)");
    int rc = ensure_attrs();
    if (rc) return rc;
    // tcgen05 block-scaled path: UE8M0 scales on both sides, 128-row weight tiles
    const bool tc_ok = !tc_disabled() && G == 0 && a_kind == WF_SCALE_E8M0 && b_kind == WF_SCALE_E8M0 &&
                       N % 128 == 0 && (K / nkc) <= wf::tc::KC_MAX && ((uintptr_t)b % 32) == 0;
    if (tc_ok) {
        const int tnkc = tc_chunks(M, N, K, wfmt == wf::FMT_FP4);
        const GemmWs Lt = gemm_ws_tc(M, N, K, tnkc);
        if (ws_bytes < Lt.total) return fail(WF_E_ARG, "workspace too small (see wf_gemm_workspace_bytes)");
        if (tnkc > 1 && gemm_shape_changed(ws, GemmShape{M, N, K, wfmt})) {
            cudaError_t e0 = cudaMemsetAsync((uint8_t *)ws + Lt.cnt, 0, Lt.part - Lt.cnt, st);
            if (e0 != cudaSuccess) return cuda_fail(e0, "cudaMemsetAsync(gemm counters)");
        }
        wf::tc::DenseArgs t;
        memset(&t, 0, sizeof(t));
        rc = weight_tensor_map(&t.tmA, b, wfmt == wf::FMT_FP4, (uint64_t)N, (uint64_t)K);
        if (rc) return rc;
        t.a = (const uint8_t *)a; t.a_s = (const uint8_t *)a_s; t.w_s = (const uint8_t *)b_s;
        t.fp4 = wfmt == wf::FMT_FP4; t.M = (int)M; t.N = (int)N; t.K = (int)K;
        t.nkc = tnkc; t.Kc = (int)(K / tnkc);
        t.out = (__nv_bfloat16 *)out; t.err = (int *)ws;
        t.cnt = (unsigned *)((uint8_t *)ws + Lt.cnt);
        t.part = (float *)((uint8_t *)ws + Lt.part);
        const int G_ = sm_count();
        if (G_ <= 0) return fail(WF_E_CUDA, "no CUDA device");
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(G_);
        lc.blockDim = dim3(wf::tc::THREADS);
        lc.dynamicSmemBytes = wf::tc::SMEM;
        lc.stream = st;
        lc.attrs = attr;
        lc.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&lc, wf::tc::k_dense_tc, t);
        if (e == cudaSuccess) counted();
        if (e == cudaSuccess) e = cudaGetLastError();
        return e == cudaSuccess ? WF_OK : cuda_fail(e, "tc gemm launch");
    }
    // tcgen05 with float32 block scales on both sides (fp8_gemm's scale_dtype float32):
    // raw per-step products, scaled and summed in registers
    const bool tc_f32 = !tc_disabled() && G == 0 && wfmt == wf::FMT_FP8 && a_kind == WF_SCALE_F32 &&
                        b_kind == WF_SCALE_F32 && N % 128 == 0 && (K / nkc) <= wf::tc::KC_MAX &&
                        ((uintptr_t)b % 32) == 0;
    if (tc_f32) {
        const int tnkc = tc_chunks(M, N, K, false);
        const GemmWs Lt = gemm_ws_tc(M, N, K, tnkc);
        if (ws_bytes < Lt.total) return fail(WF_E_ARG, "workspace too small (see wf_gemm_workspace_bytes)");
        if (tnkc > 1 && gemm_shape_changed(ws, GemmShape{M, N, K, 16 + wfmt})) {
            cudaError_t e0 = cudaMemsetAsync((uint8_t *)ws + Lt.cnt, 0, Lt.part - Lt.cnt, st);
            if (e0 != cudaSuccess) return cuda_fail(e0, "cudaMemsetAsync(gemm counters)");
        }
        wf::tc::DenseF32Args t;
        memset(&t, 0, sizeof(t));
        rc = weight_tensor_map(&t.tmA, b, false, (uint64_t)N, (uint64_t)K);
        if (rc) return rc;
        t.a = (const uint8_t *)a; t.a_s = (const float *)a_s; t.w_s = (const float *)b_s;
        t.M = (int)M; t.N = (int)N; t.K = (int)K; t.nkc = tnkc; t.Kc = (int)(K / tnkc);
        t.out = (__nv_bfloat16 *)out; t.err = (int *)ws;
        t.cnt = (unsigned *)((uint8_t *)ws + Lt.cnt);
        t.part = (float *)((uint8_t *)ws + Lt.part);
        const int G_ = sm_count();
        if (G_ <= 0) return fail(WF_E_CUDA, "no CUDA device");
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(G_);
        lc.blockDim = dim3(wf::tc::THREADS);
        lc.dynamicSmemBytes = wf::tc::F32_SMEM;
        lc.stream = st;
        lc.attrs = attr;
        lc.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&lc, wf::tc::k_dense_tc_f32, t);
        if (e == cudaSuccess) counted();
        if (e == cudaSuccess) e = cudaGetLastError();
        return e == cudaSuccess ? WF_OK : cuda_fail(e, "tc f32 gemm launch");
    }
    wf::DenseArgs d;
    d.M = (int)M; d.N = (int)N; d.K = (int)K; d.G = (int)G;
    d.wfmt = wfmt; d.a_f32 = a_kind == WF_SCALE_F32; d.b_f32 = b_kind == WF_SCALE_F32;
    d.a = (const uint8_t *)a; d.a_s = a_s; d.b = (const uint8_t *)b; d.b_s = b_s;
    d.out = (__nv_bfloat16 *)out; d.err = (int *)ws;
    d.nkc = nkc; d.Kc = (int)(K / nkc);
    d.stride = wfmt == wf::FMT_FP4 ? stride_fp4(d.Kc) : stride_fp8(d.Kc);
    d.rows = rows;
    d.cnt = (unsigned *)((uint8_t *)ws + L.cnt);
    d.part = (float *)((uint8_t *)ws + L.part);
    // this engine lays the workspace out differently: the next tcgen05 call clears it
    gemm_shape_changed(ws, GemmShape{M, N, K, -1 - wfmt});
    if (nkc > 1) {  // the workspace serves every shape: its counters start at zero per call
        cudaError_t e0 = cudaMemsetAsync((uint8_t *)ws + L.cnt, 0, L.part - L.cnt, st);
        if (e0 != cudaSuccess) return cuda_fail(e0, "cudaMemsetAsync(gemm counters)");
    }
    const int G_ = sm_count();
    if (G_ <= 0) return fail(WF_E_CUDA, "no CUDA device");
    wf::k_dense<<<G_, wf::NTHR, wf::SMEM_BYTES, st>>>(d); counted();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WF_OK : cuda_fail(e, "gemm launch");
}

int wf_fp8_gemm(const void *a, const void *a_s, int32_t a_scale_kind, const void *b,
                const void *b_s, int32_t b_scale_kind, int64_t M, int64_t N, int64_t K, void *out,
                void *workspace, size_t workspace_bytes, void *stream) {
    return dense(wf::FMT_FP8, a, a_s, a_scale_kind, b, b_s, b_scale_kind, M, N, K, 0, out,
                 workspace, workspace_bytes, (cudaStream_t)stream);
}

int wf_fp4_gemm(const void *a, const void *a_s, int32_t a_scale_kind, const void *b,
                const void *b_s, int64_t M, int64_t N, int64_t K, void *out, void *workspace,
                size_t workspace_bytes, void *stream) {
    return dense(wf::FMT_FP4, a, a_s, a_scale_kind, b, b_s, WF_SCALE_E8M0, M, N, K, 0, out,
                 workspace, workspace_bytes, (cudaStream_t)stream);
}

int wf_grouped_fp4_gemm(const void *a, const void *a_s, int32_t a_scale_kind, const void *w,
                        const void *w_s, int64_t G, int64_t N, int64_t K, void *out,
                        void *workspace, size_t workspace_bytes, void *stream) {
    if (G <= 0) return fail(WF_E_SHAPE, "G must be positive");
    return dense(wf::FMT_FP4, a, a_s, a_scale_kind, w, w_s, WF_SCALE_E8M0, G, N, K, G, out,
                 workspace, workspace_bytes, (cudaStream_t)stream);
}

int wf_fp4_scales_in_range(const uint8_t *scales, int64_t n, void *stream) {
    if (!scales || n < 0) return fail(WF_E_ARG, "null scales");
    int *dbad = nullptr;
    // load-time check: a 4-byte flag through the stream-ordered allocator
    cudaError_t e = cudaMallocAsync((void **)&dbad, 4, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocAsync");
    int host = 0;
    e = cudaMemsetAsync(dbad, 0, 4, (cudaStream_t)stream);
    if (e == cudaSuccess && n > 0) {
        wf::k_scale_range<<<296, 256, 0, (cudaStream_t)stream>>>(scales, n, dbad); counted();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(&host, dbad, 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    cudaFreeAsync(dbad, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "scale range check");
    return host ? 0 : 1;
}

}  // extern "C"
