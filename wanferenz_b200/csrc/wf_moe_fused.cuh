// wf_moe_fused.cuh - the whole MoE layer in one persistent launch on tcgen05,
// included by wf_moe.cu inside namespace wf (after wf_moe_tc.cuh, whose
// tensor-core building blocks it reuses).
//
// reference: Gate.forward, Expert.forward and MoE.forward
// (wanferenz/model/architecture.py:696-794) on the torch operators
// (wanferenz/kernels/torch_ops.py:33-108).
//
// One CTA per SM, every CTA resident for the whole launch (grid <= SM count,
// one CTA fits an SM), so CTAs may wait on one another through global memory;
// every such wait is bounded and reports kErrTimeout.  Phases:
//
//   R  router logits (fp64 sums of exact bf16 products) of this CTA's expert
//      rows for all tokens, and act_quant of the tokens t = b mod G
//   -- grid barrier --
//   S  top-k of the tokens t = b mod G (one worker warp per token)
//   -- grid barrier --
//   D  every CTA builds the dispatch tables of all tokens in its own shared
//      memory (expert counts, scan, pair lists, per-token pair lists)
//   W  four classes of tensor-core work, in this order: shared-expert w1/w3,
//      routed w1/w3, shared-expert w2, routed w2.  Each class's K steps are
//      split evenly over the CTAs (stream-K, fixed-order partial-sum fix-ups,
//      as in wf_moe_tc.cuh).  A w2 token group waits until every 128-row block
//      of its hidden state is written (a per-group counter); the last item of
//      each 256-row output block runs the ascending-expert combine.
//
// The producer warp streams the shared expert's w1/w3 weights from the first
// instruction (they depend on nothing), so the router, top-k and table phases
// run while the first weight stages arrive, and it streams w2 weights while
// the w1/w3 epilogues and fix-ups still run.  Warp roles as in wf_moe_tc.cuh:
// warps 0-3 workers (router, tables, B operand, scales, epilogues), warp 4
// TMA producer, warps 5-7 MMA issuers.
#pragma once

namespace fus {

using mtc::AM_LD;
using mtc::BSTEP;
using mtc::COL_D;
using mtc::COL_SFA;
using mtc::COL_SFB;
using mtc::GRP;
using mtc::MAX_STEPS;
using mtc::NISS;
using mtc::NT;
using mtc::NWK;
using mtc::STAGE_BYTES;
using mtc::THREADS;
using mtc::TILE_BYTES;
using mtc::W_ISS0;
using mtc::W_PROD;

constexpr int NSTG = 4;                              // weight stages (both phases)
constexpr int OFF_B = NSTG * STAGE_BYTES;            // B operand: all K steps of a token group
constexpr int B_BYTES = MAX_STEPS * BSTEP;
constexpr int OFF_BAR = OFF_B + B_BYTES;
// full[NSTG] empty[NSTG] b_ready b_free sfa_ready[2] sfa_free[2] d_ready[2] d_free[2] fin[NISS] tab
constexpr int NBAR = 2 * NSTG + 2 + 8 + NISS + 1;
constexpr int OFF_MISC = (OFF_BAR + NBAR * 8 + 127) / 128 * 128;
constexpr int OFF_PLAN = OFF_MISC + 64;     // Plan (after the misc ints)
constexpr int OFF_EX = OFF_MISC + 256;
constexpr int EX_BYTES = (128 * AM_LD + 2 * NT) * 4;
constexpr int OFF_ROUTE = OFF_EX + EX_BYTES;  // act_expert, act_off, act_tg [MAX_E + 1] each
constexpr int ROUTE_BYTES = 3 * (MAX_E + 1) * 4;
constexpr int OFF_TOK = OFF_ROUTE + ROUTE_BYTES;  // tok_pairs int16 [MAX_T * MAX_K], tok_np uint8 [MAX_T]
constexpr int TOK_BYTES = MAX_T * MAX_K * 2 + MAX_T;
constexpr int OFF_PAIR = (OFF_TOK + TOK_BYTES + 15) / 16 * 16;  // pair_tok int16, pair_w f32 [MAX_PAIRS]
constexpr int PAIR_BYTES = MAX_PAIRS * 2 + MAX_PAIRS * 4;
constexpr int SMEM = OFF_PAIR + PAIR_BYTES + 1024;  // + alignment slack
static_assert(SMEM <= 232448, "shared memory budget");
static_assert(OFF_EX % 16 == 0 && OFF_PAIR % 16 == 0, "alignment");

// Scratch of the router, top-k and table phases, inside the B-operand region
// (unused until the tables exist).
constexpr int R_SC = 0;                               // [4 warps][MAX_E] scores
constexpr int R_RIDX = R_SC + 4 * MAX_E * 4;          // int16 [MAX_T * MAX_K]
constexpr int R_POF = R_RIDX + MAX_PAIRS * 2;         // int16 [MAX_T * MAX_K]
constexpr int R_RW = R_POF + MAX_PAIRS * 2;           // f32 [MAX_T * MAX_K]
constexpr int R_CNT = R_RW + MAX_PAIRS * 4;           // int [MAX_E]
constexpr int R_BM = R_CNT + MAX_E * 4;               // u32 [MAX_E][MAX_T / 32]
constexpr int R_OFF = R_BM + MAX_E * (MAX_T / 32) * 4;  // int [MAX_E]
constexpr int R_SCAN = R_OFF + MAX_E * 4;             // u64 [4]
constexpr int R_PART = R_SCAN + 64;                   // f64 [4 warps][RROWS][RTP]
constexpr int RROWS = 2, RTP = 4;
constexpr int R_END = R_PART + 4 * RROWS * RTP * 8;
static_assert(R_END <= B_BYTES, "router scratch must fit the B region");

// misc ints
enum { M_TMEM = 0, M_ABORT = 1, M_FLAG = 2, M_NACT = 3, M_NRG = 4, M_NPAIR = 5 };

// Workspace pointers of the fused launch (beyond MoeArgs / TcArgs).
struct FArgs {
    unsigned long long *gbar;  // grid-barrier counter (monotonic)
    unsigned *hcnt;            // [groups] written 128-row blocks of each token group's h
    unsigned *cnt;             // [4][max items] stream-K arrivals per class
    float *part;               // [G][4 classes][2 slots][2 * 128 * NT]
    int max_items;
};

struct Bars {
    uint64_t *full, *empty, *b_ready, *b_free, *sfa_ready, *sfa_free, *d_ready, *d_free, *fin, *tab;
};

__device__ __forceinline__ Bars bars_at(uint8_t *base) {
    uint64_t *b = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    Bars r;
    r.full = b;
    r.empty = b + NSTG;
    r.b_ready = b + 2 * NSTG;
    r.b_free = b + 2 * NSTG + 1;
    r.sfa_ready = b + 2 * NSTG + 2;
    r.sfa_free = b + 2 * NSTG + 4;
    r.d_ready = b + 2 * NSTG + 6;
    r.d_free = b + 2 * NSTG + 8;
    r.fin = b + 2 * NSTG + 10;
    r.tab = b + 2 * NSTG + 10 + NISS;
    return r;
}

// ---------------------------------------------------------------------------
// work classes and segments
// ---------------------------------------------------------------------------
// class c: 0 shared w1/w3, 1 routed w1/w3, 2 shared w2, 3 routed w2
struct Plan {
    int nst[4], nblk[4], items[4];
    long long u0[4], u1[4], S[4];
    int nsg;  // shared token groups
};

__device__ __forceinline__ void plan_class(Plan &p, int c, int items, int G) {
    p.items[c] = items;
    p.S[c] = (long long)items * p.nst[c];
    p.u0[c] = p.S[c] * blockIdx.x / G;
    p.u1[c] = p.S[c] * (blockIdx.x + 1) / G;
}

// Classes 0 and 2 depend only on the batch size; 1 and 3 on the tables.
__device__ __forceinline__ void plan_init(Plan &p, const MoeArgs &a, int G) {
    p.nst[0] = p.nst[1] = a.D / 128;
    p.nst[2] = p.nst[3] = a.I / 128;
    p.nblk[0] = p.nblk[1] = a.I / 128;
    p.nblk[2] = p.nblk[3] = a.D / 256;
    p.nsg = cdiv(a.shT, NT);
    plan_class(p, 0, p.nsg * p.nblk[0], G);
    plan_class(p, 2, p.nsg * p.nblk[2], G);
    p.items[1] = p.items[3] = 0;
    p.S[1] = p.S[3] = p.u0[1] = p.u1[1] = p.u0[3] = p.u1[3] = 0;
}

__device__ __forceinline__ void plan_routed(Plan &p, int nrg, int G) {
    plan_class(p, 1, nrg * p.nblk[1], G);
    plan_class(p, 3, nrg * p.nblk[3], G);
}

static_assert(sizeof(Plan) <= 256 - 64, "the plan must fit the misc region");

struct Seg {
    int c, i, j0, j1, q;  // class, item, K steps [j0, j1), ordinal among this CTA's segments
};

// The segment after `sg` (sg.q < 0: the first); false when the CTA's work ends.
// `upto` bounds the classes walked (the producer walks class 0 before the tables exist).
__device__ __forceinline__ bool next_seg(const Plan &p, Seg &sg, int upto = 3) {
    int c = sg.q < 0 ? 0 : sg.c;
    long long u = sg.q < 0 ? p.u0[0] : (long long)sg.i * p.nst[c] + sg.j1;
    while (c <= upto) {
        if (u < p.u1[c]) {
            const int nst = p.nst[c];
            sg.c = c;
            sg.i = (int)(u / nst);
            sg.j0 = (int)(u - (long long)sg.i * nst);
            sg.j1 = (int)min((long long)nst, sg.j0 + (p.u1[c] - u));
            sg.q += 1;
            return true;
        }
        ++c;
        if (c <= 3) u = p.u0[c];
    }
    return false;
}

struct Tables {
    const int *act_expert, *act_off, *act_tg;
    int n_act;
};

struct TItem {
    int shared, el, blk, tok0, ntok, gid, key;
};

struct Cur {
    int c = -1, ai = 0;
};

__device__ __forceinline__ TItem decode(const MoeArgs &a, const Plan &p, const Tables &tb, Cur &cur, int c,
                                        int i) {
    TItem it;
    const int nblk = p.nblk[c];
    const int grp = i / nblk;
    it.blk = i - grp * nblk;
    if (c == 0 || c == 2) {
        it.shared = 1; it.el = 0;
        it.tok0 = a.sh0 + grp * NT; it.ntok = min(NT, a.shT - grp * NT);
        it.gid = grp;
    } else {
        if (cur.c != c) {
            int lo = 0, hi = tb.n_act - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (tb.act_tg[mid] <= grp) lo = mid; else hi = mid - 1;
            }
            cur.ai = lo;
            cur.c = c;
        }
        while (cur.ai + 1 < tb.n_act && grp >= tb.act_tg[cur.ai + 1]) ++cur.ai;
        const int tg = grp - tb.act_tg[cur.ai];
        const int p0 = tb.act_off[cur.ai], ta = tb.act_off[cur.ai + 1] - p0;
        it.shared = 0; it.el = tb.act_expert[cur.ai] - a.e0;
        it.tok0 = p0 + tg * NT; it.ntok = min(NT, ta - tg * NT);
        it.gid = p.nsg + grp;
    }
    it.key = it.gid + (c >= 2 ? (1 << 20) : 0);
    return it;
}

__device__ __forceinline__ int cta_of(long long x, long long S, int G) { return (int)(((x + 1) * G - 1) / S); }
__device__ __forceinline__ long long cta_start(int b, long long S, int G) { return S * b / G; }

__device__ __forceinline__ bool twait(uint64_t *bar, uint32_t parity, int *err, volatile int *abort,
                                      long long limit) {
    if (*abort) return false;
    if (!wf_wait(bar, parity, err, limit)) { *abort = 1; return false; }
    return true;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded spin of one thread until *p >= target; false (kErrTimeout set) when the
// bound runs out or another CTA already reported a timeout.
template <typename T, typename Load>
__device__ __forceinline__ bool spin_until(const T *p, T target, int *err, long long limit, Load load) {
    if (load(p) >= target) return true;
    const long long t0 = clock64();
    while (load(p) < target) {
        if (*reinterpret_cast<volatile int *>(err) & kErrTimeout) return false;
        if (clock64() - t0 > limit) {
            atomicOr(err, kErrTimeout);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Grid barrier of the worker threads (128 per CTA): every CTA's earlier global
// writes are visible to every CTA after it.  The counter only grows: barrier n
// of a launch completes at the next multiple of G.
__device__ __forceinline__ bool grid_barrier(const FArgs &f, int *err, long long limit, int G,
                                             volatile int *flag) {
    bar_sync(2, NWK);
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long old = atomicAdd(f.gbar, 1ull);
        const unsigned long long target = (old / (unsigned long long)G + 1ull) * (unsigned long long)G;
        *flag = spin_until(f.gbar, target, err, limit, ld_acquire_u64) ? 1 : 0;
    }
    bar_sync(2, NWK);
    return *flag != 0;
}

// ---------------------------------------------------------------------------
// expert parallelism over peer memory
// ---------------------------------------------------------------------------
// Every rank's CTA 0 (after the rank's own grid barrier) publishes this launch's
// epoch in every rank's dispatch flags; each CTA then waits (bounded) until all
// ranks' flags carry it: every rank's tokens and routing are in this rank's buffer.
__device__ __forceinline__ bool ep_dispatch_handshake(const MoeArgs &a, unsigned epoch, volatile int *flag) {
    bar_sync(2, NWK);
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0) {
            __threadfence_system();
            for (int p = 0; p < a.ep_world; ++p) st_release_sys_u32(a.ep_flags[p] + a.ep_rank, epoch);
        }
        bool ok = true;
        for (int p = 0; p < a.ep_world && ok; ++p)
            ok = spin_until(a.ep_flags[a.ep_rank] + p, epoch, a.err, a.wait_limit, ld_acquire_sys_u32);
        *flag = ok ? 1 : 0;
    }
    bar_sync(2, NWK);
    return *flag != 0;
}

// After a 256-row output block's combine wrote its rows to their owners: the CTA
// that completes the last block publishes the epoch in every rank's combine flags.
__device__ __forceinline__ void ep_block_done(const MoeArgs &a, unsigned epoch, int nblocks, int bar_id) {
    __threadfence_system();
    bar_sync(bar_id, NWK);
    if (threadIdx.x == 0) {
        const unsigned old = atomicAdd(a.ep_done, 1u);
        if (old == (unsigned)nblocks - 1) {
            *a.ep_done = 0u;
            __threadfence_system();
            for (int p = 0; p < a.ep_world; ++p)
                st_release_sys_u32(a.ep_flags[p] + EP_MAX_RANKS + a.ep_rank, epoch);
        }
    }
}

// act_quant of this rank's tokens t = b, b + G, ... (rows ep_rank * Tr + t of the
// gathered batch), written to every rank's buffer.
__device__ void quantize_tokens_ep(const MoeArgs &a) {
    const int lane = threadIdx.x & 31;
    const int nb = a.D / 128;
    for (int t = blockIdx.x; t < a.Tr; t += gridDim.x) {
        const size_t grow = (size_t)a.ep_rank * a.Tr + t;
        for (int b = 0; b < nb; ++b) {
            const uint2 u = __ldg(reinterpret_cast<const uint2 *>(a.x + (size_t)t * a.D + b * 128 + 4 * lane));
            const float v0 = bf16_bits_to_f32(u.x & 0xffffu), v1 = bf16_bits_to_f32(u.x >> 16);
            const float v2 = bf16_bits_to_f32(u.y & 0xffffu), v3 = bf16_bits_to_f32(u.y >> 16);
            float m = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float s = round_scale_e8(fmaxf(m, 1e-4f), 1);
            const float inv = 1.0f / s;  // exact: s is a power of two
            auto qz = [&](float v) { return fminf(fmaxf(v * inv, -448.f), 448.f); };
            const uint32_t q = (uint32_t)f32x2_to_e4m3x2(qz(v0), qz(v1)) | ((uint32_t)f32x2_to_e4m3x2(qz(v2), qz(v3)) << 16);
            const uint8_t sb = (uint8_t)((__float_as_uint(s) >> 23) & 0xffu);
            for (int p = 0; p < a.ep_world; ++p) {
                *reinterpret_cast<uint32_t *>(a.ep_xq[p] + grow * a.D + b * 128 + 4 * lane) = q;
                if (lane == 0) a.ep_xs[p][grow * nb + b] = sb;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// phase R: router logits of this CTA's expert rows (e = b + r*G), all tokens
// ---------------------------------------------------------------------------
__device__ void router_rows(const MoeArgs &a, uint8_t *scr, int G) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = a.E, D = a.D, T = a.ep ? a.Tr : a.T;  // the tokens routed on this rank
    const int nrows = ((int)blockIdx.x < E) ? cdiv(E - (int)blockIdx.x, G) : 0;
    const int quarter = D / 4;  // warp w sums quarter w of every row
    double *part = reinterpret_cast<double *>(scr + R_PART);  // [warp][row][token]
    constexpr int KU = 4;  // 256-element chunks of a lane (quarter <= 1024)
    for (int r0 = 0; r0 < nrows; r0 += RROWS) {
        float wf[RROWS][KU][8];
#pragma unroll
        for (int rr = 0; rr < RROWS; ++rr) {
            const bool rv = r0 + rr < nrows;
            const __nv_bfloat16 *wrow =
                a.gate_w + (size_t)(rv ? (int)blockIdx.x + (r0 + rr) * G : 0) * D + warp * quarter;
            uint4 wu[KU];
#pragma unroll
            for (int u = 0; u < KU; ++u) {
                const int k = lane * 8 + u * 256;
                wu[u] = (rv && k < quarter) ? ldg128(wrow + k) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < KU; ++u) {
                const uint32_t wv[4] = {wu[u].x, wu[u].y, wu[u].z, wu[u].w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    wf[rr][u][2 * c] = bf16_bits_to_f32(wv[c] & 0xffffu);
                    wf[rr][u][2 * c + 1] = bf16_bits_to_f32(wv[c] >> 16);
                }
            }
        }
        for (int t0 = 0; t0 < T; t0 += RTP) {
            uint4 xu[KU][RTP];
#pragma unroll
            for (int u = 0; u < KU; ++u)
#pragma unroll
                for (int t = 0; t < RTP; ++t) {
                    const int k = lane * 8 + u * 256;
                    xu[u][t] = (k < quarter && t0 + t < T)
                                   ? ldg128(a.x + (size_t)(t0 + t) * D + warp * quarter + k)
                                   : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
            for (int rr = 0; rr < RROWS; ++rr) {
                if (r0 + rr >= nrows) break;
                double acc[RTP];
#pragma unroll
                for (int t = 0; t < RTP; ++t) {
                    acc[t] = 0.0;
#pragma unroll
                    for (int u = 0; u < KU; ++u) {
                        const uint32_t xv[4] = {xu[u][t].x, xu[u][t].y, xu[u][t].z, xu[u][t].w};
                        double s = 0.0;
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            // bf16 x bf16 products are exact in fp32
                            s += (double)(wf[rr][u][2 * c] * bf16_bits_to_f32(xv[c] & 0xffffu));
                            s += (double)(wf[rr][u][2 * c + 1] * bf16_bits_to_f32(xv[c] >> 16));
                        }
                        acc[t] += s;
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
                }
                if (lane == 0) {
#pragma unroll
                    for (int t = 0; t < RTP; ++t) part[(warp * RROWS + rr) * RTP + t] = acc[t];
                }
            }
            bar_sync(2, NWK);
            if (threadIdx.x < RROWS * RTP) {
                const int rr = threadIdx.x / RTP, t = threadIdx.x % RTP;
                if (r0 + rr < nrows && t0 + t < T) {
                    // the four quarters in a fixed order
                    const double v = part[(0 * RROWS + rr) * RTP + t] + part[(1 * RROWS + rr) * RTP + t] +
                                     part[(2 * RROWS + rr) * RTP + t] + part[(3 * RROWS + rr) * RTP + t];
                    a.logits[(size_t)(t0 + t) * E + blockIdx.x + (r0 + rr) * G] = (float)v;
                }
            }
            bar_sync(2, NWK);
        }
    }
}

// ---------------------------------------------------------------------------
// phase D: the dispatch tables of all tokens, in this CTA's shared memory
// (the steps of topk_dispatch, on the 128 worker threads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long scan128_u64(unsigned long long v, unsigned long long *ws,
                                                          unsigned long long &tot) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) ws[warp] = v;
    bar_sync(2, NWK);
    unsigned long long before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const unsigned long long x = ws[w];
        if (w < warp) before += x;
        all += x;
    }
    bar_sync(2, NWK);
    tot = all;
    return v + before;  // inclusive
}

__device__ void build_tables(const MoeArgs &a, uint8_t *base, uint8_t *scr, volatile int *misc) {
    const int tid = threadIdx.x;
    const int T = a.T, E = a.E, K = a.topk, El = a.El;
    int16_t *ridx_s = reinterpret_cast<int16_t *>(scr + R_RIDX);
    int16_t *pof_s = reinterpret_cast<int16_t *>(scr + R_POF);
    float *rw_s = reinterpret_cast<float *>(scr + R_RW);
    int *cnt_s = reinterpret_cast<int *>(scr + R_CNT);
    uint32_t *bm = reinterpret_cast<uint32_t *>(scr + R_BM);
    int *off_s = reinterpret_cast<int *>(scr + R_OFF);
    unsigned long long *scan_ws = reinterpret_cast<unsigned long long *>(scr + R_SCAN);
    int *act_expert = reinterpret_cast<int *>(base + OFF_ROUTE);
    int *act_off = act_expert + (MAX_E + 1);
    int *act_tg = act_off + (MAX_E + 1);
    int16_t *tp_s = reinterpret_cast<int16_t *>(base + OFF_TOK);
    uint8_t *np_s = base + OFF_TOK + MAX_T * MAX_K * 2;
    int16_t *pt_s = reinterpret_cast<int16_t *>(base + OFF_PAIR);
    float *pw_s = reinterpret_cast<float *>(base + OFF_PAIR + MAX_PAIRS * 2);
    const int TW = (T + 31) >> 5;
    // 1. the routing of every token: this launch's top-k, or given by the caller
    for (int slot = tid; slot < T * K; slot += NWK) {
        long long e;
        float w;
        if (a.given) {
            e = __ldg(a.in_idx + slot);
            w = __ldg(a.in_w + slot);
        } else {
            e = __ldcg(a.ridx + slot);
            w = __ldcg(a.rw + slot);
        }
        if (e < 0 || e >= E) { atomicOr(a.err, kErrExpertId); e = 0; }
        ridx_s[slot] = (int16_t)e;
        rw_s[slot] = w;
        pof_s[slot] = -1;
    }
    for (int i = tid; i < El; i += NWK) cnt_s[i] = 0;
    for (int i = tid; i < El * TW; i += NWK) bm[i] = 0u;
    bar_sync(2, NWK);
    // 2. keep flags (a duplicated expert keeps its last slot), counts, token bitmaps
    for (int slot = tid; slot < T * K; slot += NWK) {
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
    bar_sync(2, NWK);
    // 3. scan over local experts (4 per thread): pair offset | token groups | active index
    constexpr int EPT = MAX_E / NWK;
    auto pack = [](int c) -> unsigned long long {
        return (unsigned long long)c | ((unsigned long long)cdiv(c, NT) << 16) | ((unsigned long long)(c > 0) << 32);
    };
    unsigned long long v[EPT], mine = 0;
    int cs[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int el = EPT * tid + k;
        cs[k] = el < El ? cnt_s[el] : 0;
        v[k] = pack(cs[k]);
        mine += v[k];
    }
    unsigned long long tot;
    unsigned long long ex = scan128_u64(mine, scan_ws, tot) - mine;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int el = EPT * tid + k;
        if (el < El) {
            const int off = (int)(ex & 0xffff), tg = (int)((ex >> 16) & 0xffff), n = (int)((ex >> 32) & 0xffff);
            off_s[el] = off;
            if (cs[k]) {
                act_expert[n] = a.e0 + el;
                act_off[n] = off;
                act_tg[n] = tg;
            }
        }
        ex += v[k];
    }
    if (tid == NWK - 1) {
        const int off = (int)(tot & 0xffff), tg = (int)((tot >> 16) & 0xffff), n = (int)((tot >> 32) & 0xffff);
        act_off[n] = off;
        act_tg[n] = tg;
        misc[M_NACT] = n;
        misc[M_NRG] = tg;
        misc[M_NPAIR] = off;
    }
    bar_sync(2, NWK);
    // 4. pairs: expert ascending, token ascending within an expert
    for (int slot = tid; slot < T * K; slot += NWK) {
        if (pof_s[slot] != -2) continue;
        const int t = slot / K;
        const int el = ridx_s[slot] - a.e0;
        const uint32_t *row = bm + el * TW;
        int rank = __popc(row[t >> 5] & ((1u << (t & 31)) - 1u));
        for (int w = 0; w < (t >> 5); ++w) rank += __popc(row[w]);
        const int p = off_s[el] + rank;
        pt_s[p] = (int16_t)t;
        pw_s[p] = rw_s[slot];
        pof_s[slot] = (int16_t)p;
    }
    bar_sync(2, NWK);
    // 5. each token's pairs in ascending expert order
    for (int t = tid; t < T; t += NWK) {
        int n = 0;
        for (int j = 0; j < K; ++j) {
            const int p = pof_s[t * K + j];
            if (p < 0) continue;
            const int e = ridx_s[t * K + j];
            int rank = 0;
            for (int j2 = 0; j2 < K; ++j2) rank += (pof_s[t * K + j2] >= 0 && ridx_s[t * K + j2] < e) ? 1 : 0;
            tp_s[t * K + rank] = (int16_t)p;
            ++n;
        }
        np_s[t] = (uint8_t)n;
    }
    bar_sync(2, NWK);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS, 1) k_moe_fused(const __grid_constant__ MoeArgs a,
                                                          const __grid_constant__ mtc::TcArgs t,
                                                          const __grid_constant__ FArgs f) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Bars B = bars_at(base);
    volatile int *misc = reinterpret_cast<volatile int *>(base + OFF_MISC);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(base + OFF_MISC) + M_TMEM;
    volatile int *abort = misc + M_ABORT;
    volatile int *flag = misc + M_FLAG;
    float *ex = reinterpret_cast<float *>(base + OFF_EX);
    uint8_t *scr = base + OFF_B;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTG; ++s) { mbar_init(B.full + s, 1); mbar_init(B.empty + s, NISS); }
        mbar_init(B.b_ready, 4);
        mbar_init(B.b_free, NISS);
        for (int j = 0; j < 2; ++j) {
            mbar_init(B.sfa_ready + j, 4); mbar_init(B.sfa_free + j, NISS);
            mbar_init(B.d_ready + j, NISS); mbar_init(B.d_free + j, 4);
        }
        for (int j = 0; j < NISS; ++j) mbar_init(B.fin + j, 1);
        mbar_init(B.tab, 1);
        *abort = 0;
        *flag = 0;
        plan_init(*reinterpret_cast<Plan *>(base + OFF_PLAN), a, G);
        fence_mbar_init();
    }
    if (warp == W_PROD) { tc::tmem_alloc(tmem_slot, 512); tc::tmem_relinquish(); }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tm = *tmem_slot;
    pdl_launch_dependents();

    Plan &p = *reinterpret_cast<Plan *>(base + OFF_PLAN);
    Tables tb;
    tb.act_expert = reinterpret_cast<const int *>(base + OFF_ROUTE);
    tb.act_off = tb.act_expert + (MAX_E + 1);
    tb.act_tg = tb.act_off + (MAX_E + 1);
    tb.n_act = 0;
    const int16_t *tp_s = reinterpret_cast<const int16_t *>(base + OFF_TOK);
    const uint8_t *np_s = base + OFF_TOK + MAX_T * MAX_K * 2;
    const int16_t *pt_s = reinterpret_cast<const int16_t *>(base + OFF_PAIR);
    const float *pw_s = reinterpret_cast<const float *>(base + OFF_PAIR + MAX_PAIRS * 2);
    const int D = a.D, I = a.I;

    // the tables exist (mbarrier `tab`; the routed classes are planned in `p`)
    auto await_tables = [&]() -> bool {
        if (!twait(B.tab, 0, a.err, abort, a.wait_limit)) return false;
        tb.n_act = misc[M_NACT];
        return true;
    };

    if (warp == W_PROD) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = tc::policy_evict_first();
            Cur cur;
            Seg sg{0, 0, 0, 0, -1};
            int gs = 0, st = 0, lap = 0;
            bool have_tab = false;
            while (!*abort) {
                if (!next_seg(p, sg, have_tab ? 3 : 0)) {
                    if (have_tab) break;
                    // class 0 ran out: the later classes need the tables
                    if (!await_tables()) break;
                    have_tab = true;
                    continue;
                }
                const TItem it = decode(a, p, tb, cur, sg.c, sg.i);
                const bool ph2 = sg.c < 2;
                const uint32_t tx = it.shared ? STAGE_BYTES : STAGE_BYTES / 2;
                bool ok = true;
                for (int j = sg.j0; j < sg.j1; ++j, ++gs, lap += (st + 1 == NSTG), st = (st + 1 == NSTG) ? 0 : st + 1) {
                    if (gs >= NSTG && !twait(B.empty + st, (lap - 1) & 1, a.err, abort, a.wait_limit)) { ok = false; break; }
                    uint8_t *dst = base + st * STAGE_BYTES;
                    mbar_arrive_expect_tx(B.full + st, tx);
                    if (ph2) {
                        if (it.shared) tc::tma_load_3d_hint(dst, &t.m_s13, j * 128, it.blk * 128, 0, B.full + st, pol);
                        else tc::tma_load_3d_hint(dst, &t.m_r13, j * 128, it.blk * 128, 2 * it.el, B.full + st, pol);
                    } else {
                        if (it.shared) tc::tma_load_2d_hint(dst, &t.m_s2, j * 128, it.blk * 256, B.full + st, pol);
                        else tc::tma_load_2d_hint(dst, &t.m_r2, j * 128, it.el * D + it.blk * 256, B.full + st, pol);
                    }
                }
                if (!ok) break;
            }
            // every issued copy lands before the CTA may exit
            for (int k = 0; k < NSTG && k < gs; ++k) {
                const int g = gs - 1 - k;
                wf_wait(B.full + g % NSTG, (g / NSTG) & 1, a.err);
            }
        }
    } else if (warp >= W_ISS0) {
        // ------------------------------------------------------------ MMA issuers
        const int ii = warp - W_ISS0;
        if (lane == 0) {
            if (await_tables()) {
                Cur cur;
                Seg sg{0, 0, 0, 0, -1};
                int gs = 0, gi = 0, nb = 0, key = -1;
                int st = 0, lap = 0;
                const uint64_t a0 = tc::smem_desc_sw128(base);
                const uint64_t b0 = tc::smem_desc_sw128(base + OFF_B);
                bool more = next_seg(p, sg);
                while (more && !*abort) {
                    const TItem it = decode(a, p, tb, cur, sg.c, sg.i);
                    const int buf = sg.q & 1;
                    if (it.key != key) {
                        if (!twait(B.b_ready, nb & 1, a.err, abort, a.wait_limit)) break;
                        ++nb;
                        key = it.key;
                    }
                    if (sg.q >= 2 && !twait(B.d_free + buf, ((sg.q >> 1) - 1) & 1, a.err, abort, a.wait_limit)) break;
                    tc::fence_after_sync();
                    const int afmt = it.shared ? 0 : 5;
                    const uint32_t id0 = tc::idesc_mxf8f6f4(afmt, 0, NT, 0), id1 = tc::idesc_mxf8f6f4(afmt, 0, NT, 1);
                    const uint32_t id2 = tc::idesc_mxf8f6f4(afmt, 0, NT, 2), id3 = tc::idesc_mxf8f6f4(afmt, 0, NT, 3);
                    const uint32_t dcol = tm + COL_D + (uint32_t)((ii * 2 + buf) * 2 * NT);
                    bool first = true, ok = true;
                    int own = 0;
                    for (int j = sg.j0; j < sg.j1; ++j, ++gs, own = (own + 1 == NISS) ? 0 : own + 1,
                             lap += (st + 1 == NSTG), st = (st + 1 == NSTG) ? 0 : st + 1) {
                        const int gj = j & (GRP - 1);
                        if (j == sg.j0 || gj == 0) {
                            if (!twait(B.sfa_ready + (gi & 1), (gi >> 1) & 1, a.err, abort, a.wait_limit)) { ok = false; break; }
                        }
                        // every issuer waits for every stage use (see wf_moe_tc.cuh)
                        if (!twait(B.full + st, lap & 1, a.err, abort, a.wait_limit)) { ok = false; break; }
                        if (own != ii) {
                            mbar_arrive(B.empty + st);
                        } else {
                            tc::fence_after_sync();
                            const uint64_t ad = a0 + (uint64_t)((st * STAGE_BYTES) >> 4);
                            const uint64_t bd = b0 + (uint64_t)((j * BSTEP) >> 4);
                            const uint32_t sfa = tm + COL_SFA + (uint32_t)((gi & 1) * (GRP * 8) + gj * 8);
                            const uint32_t sfb = tm + COL_SFB + (uint32_t)(4 * j);
#pragma unroll
                            for (int tt = 0; tt < 2; ++tt) {
                                const uint64_t at = ad + (uint64_t)((tt * TILE_BYTES) >> 4);
                                const uint32_t dc = dcol + (uint32_t)(tt * NT), sa = sfa + (uint32_t)(4 * tt);
                                tc::mma_mxf8f6f4(dc, at + 0, bd + 0, id0, sa, sfb, first ? 0u : 1u);
                                tc::mma_mxf8f6f4(dc, at + 2, bd + 2, id1, sa, sfb, 1u);
                                tc::mma_mxf8f6f4(dc, at + 4, bd + 4, id2, sa, sfb, 1u);
                                tc::mma_mxf8f6f4(dc, at + 6, bd + 6, id3, sa, sfb, 1u);
                            }
                            first = false;
                            tc::commit(B.empty + st);
                        }
                        if (gj == GRP - 1 || j == sg.j1 - 1) {
                            tc::commit(B.sfa_free + (gi & 1));
                            ++gi;
                        }
                    }
                    if (!ok) break;
                    tc::commit(B.d_ready + buf);
                    const int key_now = it.key;
                    more = next_seg(p, sg);
                    if (!more) {
                        tc::commit(B.b_free);
                    } else {
                        Cur c2 = cur;
                        if (decode(a, p, tb, c2, sg.c, sg.i).key != key_now) tc::commit(B.b_free);
                    }
                }
            }
            // all of this thread's MMAs complete before TMEM is released
            tc::commit(B.fin + ii);
            wf_wait(B.fin + ii, 0, a.err);
        }
    } else {
        // ------------------------------------------------------------ workers
        const int tid = threadIdx.x;
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        const int row = 32 * warp + lane;
        bool dead = false;
        // everything below reads what the previous kernel on the stream wrote
        pdl_wait();
        // expert parallelism: this forward's epoch (the previous one's finish advanced the counter)
        const unsigned ep_epoch = a.ep ? __ldcg(a.ep_flags[a.ep_rank] + EP_CTR) + 1u : 0u;
        if (blockIdx.x == 0) {
            // this launch's h-ready counters start at zero (before the first barrier)
            const int ngr = p.nsg + min(a.El, a.T * a.topk) + cdiv(a.T * a.topk, NT);
            for (int k = tid; k < ngr; k += NWK) f.hcnt[k] = 0u;
        }
        // ---- R: router logits of this CTA's rows; act_quant of tokens b, b + G, ...
        if (!a.given) router_rows(a, scr, G);
        if (warp == 0) {
            if (a.ep) quantize_tokens_ep(a);
            else quantize_tokens_warp(a);
        }
        if (!grid_barrier(f, a.err, a.wait_limit, G, flag)) dead = true;
        // ---- S: top-k of tokens t = b mod G, one worker warp each (expert
        // parallelism: this rank's tokens, their routing written to every rank)
        if (!dead && !a.given) {
            float *sc_w = reinterpret_cast<float *>(scr + R_SC) + warp * MAX_E;
            int16_t *ridx_s = reinterpret_cast<int16_t *>(scr + R_RIDX);
            int16_t *pof_s = reinterpret_cast<int16_t *>(scr + R_POF);
            float *rw_s = reinterpret_cast<float *>(scr + R_RW);
            const int Tq = a.ep ? a.Tr : a.T;
            for (int tk = blockIdx.x + warp * G; tk < Tq; tk += 4 * G) {
                if (a.E <= 256) topk_token<8>(topk_in(a), tk, lane, sc_w, ridx_s, pof_s, rw_s, false);
                else topk_token<MAX_E / 32>(topk_in(a), tk, lane, sc_w, ridx_s, pof_s, rw_s, false);
                if (lane < a.topk) {
                    const int e = ridx_s[tk * a.topk + lane];
                    const float w = rw_s[tk * a.topk + lane];
                    if (a.ep) {
                        const size_t g = ((size_t)a.ep_rank * a.Tr + tk) * a.topk + lane;
                        for (int pr = 0; pr < a.ep_world; ++pr) {
                            a.ep_ridx[pr][g] = e;
                            a.ep_rw[pr][g] = w;
                        }
                    } else {
                        a.ridx[tk * a.topk + lane] = e;
                        a.rw[tk * a.topk + lane] = w;
                    }
                }
            }
            if (a.ep) __threadfence_system();
            if (!grid_barrier(f, a.err, a.wait_limit, G, flag)) dead = true;
            if (!dead && a.ep && !ep_dispatch_handshake(a, ep_epoch, flag)) dead = true;
        }
        // ---- D: tables, then release the producer and the issuers
        if (!dead) build_tables(a, base, scr, misc);
        if (tid == 0 && !dead) plan_routed(p, misc[M_NRG], G);
        tc::fence_before_sync();
        bar_sync(2, NWK);
        if (tid == 0) {
            if (dead) *abort = 1;
            mbar_arrive(B.tab);
        }
        if (!dead) tb.n_act = misc[M_NACT];
        const int ngroups = p.nsg + (dead ? 0 : misc[M_NRG]);
        if (!dead && ngroups == 0) {
            // no work at all (a routed-only call whose shard got no tokens): the
            // combine still writes every row block (zeros)
            for (int rb = blockIdx.x; rb < D / 256; rb += G) {
                combine_rows_v8<NWK>(a, rb * 256, 256, np_s, tp_s);
                if (a.ep) ep_block_done(a, ep_epoch, D / 256, 2);
            }
        }

        auto wwait = [&](uint64_t *bar, uint32_t parity) -> bool {
            const bool ok = twait(bar, parity, a.err, abort, a.wait_limit);
            if (mtc::bar_or(1, NWK, !ok)) dead = true;
            return !dead;
        };

        Cur cur, cur_e;
        Seg sg{0, 0, 0, 0, -1};
        int gi = 0, nb = 0, key = -1;
        uint8_t *Bsm = base + OFF_B;

        auto epilogue = [&](const Seg &e) {
            const TItem it = decode(a, p, tb, cur_e, e.c, e.i);
            const int buf = e.q & 1;
            const int nst = p.nst[e.c];
            if (!wwait(B.d_ready + buf, (e.q >> 1) & 1)) return;
            tc::fence_after_sync();
            float g[NT], u[NT];
            const int nsteps = e.j1 - e.j0;
#pragma unroll
            for (int ii = 0; ii < NISS; ++ii) {
                if (ii > 0 && nsteps <= ii) break;
                uint32_t v0[NT], v1[NT];
                const uint32_t col = COL_D + (uint32_t)((ii * 2 + buf) * 2 * NT);
                tc::tmem_ld16(tm + lane_base + col, v0);
                tc::tmem_ld16(tm + lane_base + col + NT, v1);
                tc::tmem_wait_ld();
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    if (ii == 0) { g[n] = __uint_as_float(v0[n]); u[n] = __uint_as_float(v1[n]); }
                    else { g[n] += __uint_as_float(v0[n]); u[n] += __uint_as_float(v1[n]); }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(B.d_free + buf);
            const int ntok = it.ntok;
            if (!(e.j0 == 0 && e.j1 == nst)) {
                // stream-K: partials to this CTA's slot of the class; the last segment of
                // the item to arrive sums every segment's partials in CTA order
                const long long S = p.S[e.c];
                const long long is = (long long)e.i * nst;
                const int slot = (blockIdx.x * 4 + e.c) * 2 + (p.u0[e.c] >= is ? 0 : 1);
                float4 *ps = reinterpret_cast<float4 *>(f.part + (size_t)slot * (2 * 128 * NT));
#pragma unroll
                for (int c = 0; c < NT / 4; ++c) {
                    if (4 * c >= ntok) break;
                    ps[c * 128 + row] = make_float4(g[4 * c], g[4 * c + 1], g[4 * c + 2], g[4 * c + 3]);
                    ps[(NT / 4 + c) * 128 + row] = make_float4(u[4 * c], u[4 * c + 1], u[4 * c + 2], u[4 * c + 3]);
                }
                __threadfence();
                bar_sync(1, NWK);
                unsigned *cnt = f.cnt + (size_t)e.c * f.max_items + e.i;
                const int blo = cta_of(is, S, G), bhi = cta_of(is + nst - 1, S, G);
                if (tid == 0) {
                    int nseg = 0;
                    for (int b = blo; b <= bhi; ++b) nseg += cta_start(b + 1, S, G) > cta_start(b, S, G);
                    const unsigned old = atomicAdd(cnt, 1u);
                    *flag = old == (unsigned)(nseg - 1);
                }
                bar_sync(1, NWK);
                const int last = *flag;
                bar_sync(1, NWK);
                if (!last) return;
                __threadfence();
#pragma unroll
                for (int n = 0; n < NT; ++n) { g[n] = 0.f; u[n] = 0.f; }
#pragma unroll 2
                for (int b = blo; b <= bhi; ++b) {
                    const long long ub = cta_start(b, S, G);
                    if (cta_start(b + 1, S, G) <= ub) continue;
                    const float4 *pp = reinterpret_cast<const float4 *>(
                        f.part + (size_t)((b * 4 + e.c) * 2 + (ub >= is ? 0 : 1)) * (2 * 128 * NT));
                    float4 vg[NT / 4], vu[NT / 4];
#pragma unroll
                    for (int c = 0; c < NT / 4; ++c) {
                        if (4 * c >= ntok) break;
                        vg[c] = __ldcg(pp + c * 128 + row);
                        vu[c] = __ldcg(pp + (NT / 4 + c) * 128 + row);
                    }
#pragma unroll
                    for (int c = 0; c < NT / 4; ++c) {
                        if (4 * c >= ntok) break;
                        g[4 * c] += vg[c].x; g[4 * c + 1] += vg[c].y; g[4 * c + 2] += vg[c].z; g[4 * c + 3] += vg[c].w;
                        u[4 * c] += vu[c].x; u[4 * c + 1] += vu[c].y; u[4 * c + 2] += vu[c].z; u[4 * c + 3] += vu[c].w;
                    }
                }
                if (tid == 0) *cnt = 0u;
            }
            if (e.c < 2) {
                // SwiGLU (architecture.py:733-741), route weight, bf16, then act_quant of
                // this 128-row block of h (per-token amax through a shared-memory transpose)
                float h[NT];
#pragma unroll
                for (int c = 0; c < NT / 4; ++c) {
                    if (4 * c >= ntok) break;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int n = 4 * c + k;
                        float hv = swiglu(g[n], u[n], a.swiglu_limit);
                        if (!it.shared) hv = (n < ntok ? pw_s[it.tok0 + n] : 0.f) * hv;
                        h[n] = n < ntok ? bf16r(hv) : 0.f;
                    }
                    *reinterpret_cast<float4 *>(ex + row * AM_LD + 4 * c) =
                        make_float4(fabsf(h[4 * c]), fabsf(h[4 * c + 1]), fabsf(h[4 * c + 2]), fabsf(h[4 * c + 3]));
                }
                bar_sync(1, NWK);
                float *inv_s = ex + 128 * AM_LD;
                uint32_t *sb_s = reinterpret_cast<uint32_t *>(inv_s + NT);
                {
                    const int n = tid >> 3, part = tid & 7;
                    float m = 0.f;
                    if (n < ntok) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) m = fmaxf(m, ex[(part + 8 * i) * AM_LD + n]);
                    }
#pragma unroll
                    for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                    if (part == 0 && n < ntok) {
                        const float sc = round_scale_e8(fmaxf(m, 1e-4f), 1);
                        inv_s[n] = 1.0f / sc;  // exact: sc is a power of two
                        sb_s[n] = (__float_as_uint(sc) >> 23) & 0xffu;
                    }
                }
                bar_sync(1, NWK);
                uint8_t *dq = it.shared ? t.sq : t.hq;
                uint8_t *ds = it.shared ? t.sqs : t.hqs;
                const int ib = I / 128;
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    if (n >= ntok) break;
                    const float qv = fminf(fmaxf(h[n] * inv_s[n], -448.f), 448.f);
                    dq[(size_t)(it.tok0 + n) * I + it.blk * 128 + row] = mtc::e4m3_byte(qv);
                }
                if (tid < ntok) ds[(size_t)(it.tok0 + tid) * ib + it.blk] = (uint8_t)sb_s[tid];
                __threadfence();
                bar_sync(1, NWK);  // the tile is reused by the next epilogue
                if (tid == 0) atomicAdd(f.hcnt + it.gid, 1u);  // one more block of this group's h
            } else {
                __nv_bfloat16 *dst = it.shared ? a.os : a.o;
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    if (n >= ntok) break;
                    const size_t o = (size_t)(it.tok0 + n) * D + it.blk * 256 + row;
                    dst[o] = __float2bfloat16_rn(g[n]);
                    dst[o + 128] = __float2bfloat16_rn(u[n]);
                }
                // combine of this 256-row block once every token group has written it
                __threadfence();
                bar_sync(1, NWK);
                if (tid == 0) {
                    const unsigned old = atomicAdd(a.cnt_rb + it.blk, 1u);
                    *flag = old == (unsigned)ngroups - 1;
                }
                bar_sync(1, NWK);
                const int last = *flag;
                bar_sync(1, NWK);
                if (last) {
                    __threadfence();
                    combine_rows_v8<NWK>(a, it.blk * 256, 256, np_s, tp_s);
                    if (tid == 0) a.cnt_rb[it.blk] = 0u;
                    if (a.ep) ep_block_done(a, ep_epoch, D / 256, 1);
                }
            }
        };

        Seg prev{0, 0, 0, 0, -1};
        bool have_prev = false;
        while (!dead && next_seg(p, sg)) {
            const TItem it = decode(a, p, tb, cur, sg.c, sg.i);
            const int nst = p.nst[sg.c];
            const int K = sg.c < 2 ? D : I;
            if (it.key != key) {
                if (sg.c >= 2) {
                    // w2 of this group reads its whole h: first the pending w1/w3 epilogue
                    // (it may write a block of that h), then wait for every block
                    if (have_prev && prev.c < 2) {
                        epilogue(prev);
                        have_prev = false;
                        if (dead) break;
                    }
                    if (tid == 0)
                        *flag = spin_until(f.hcnt + it.gid, (unsigned)(I / 128), a.err, a.wait_limit, ld_acquire_u32);
                    bar_sync(1, NWK);
                    const int ok = *flag;
                    bar_sync(1, NWK);
                    if (!ok) { *abort = 1; dead = true; break; }
                }
                if (nb > 0 && !wwait(B.b_free, (nb - 1) & 1)) break;
                const uint8_t *src0;
                const uint8_t *sc0;
                size_t rstride, sstride;
                if (sg.c < 2) { src0 = t.xq; sc0 = t.xs; rstride = D; sstride = D / 128; }
                else if (it.shared) { src0 = t.sq; sc0 = t.sqs; rstride = I; sstride = I / 128; }
                else { src0 = t.hq; sc0 = t.hqs; rstride = I; sstride = I / 128; }
                auto tok_row = [&](int n) -> size_t {
                    if (sg.c == 1) return (size_t)pt_s[it.tok0 + n];
                    return (size_t)(it.tok0 + n);
                };
                const int nchunk = it.ntok * nst * 8;
                for (int c0 = tid; c0 < nchunk; c0 += 8 * NWK) {
                    uint4 v[8];
                    int dsto[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int c = c0 + k * NWK;
                        dsto[k] = -1;
                        if (c < nchunk) {
                            const int n = c / (nst * 8), rem = c - n * (nst * 8);
                            const int s = rem >> 3, ch = rem & 7;
                            v[k] = ldcg128(src0 + tok_row(n) * rstride + s * 128 + ch * 16);
                            dsto[k] = s * BSTEP + (int)tc::sw128_offset(n, ch);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (dsto[k] >= 0) *reinterpret_cast<uint4 *>(Bsm + dsto[k]) = v[k];
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                {
                    const bool tv = lane < it.ntok;
                    const uint8_t *sr = tv ? sc0 + tok_row(lane) * sstride : nullptr;
                    for (int s = 0; s < nst; ++s) {
                        const uint32_t w = tv ? 0x01010101u * (uint32_t)__ldcg(sr + s) : 0x7f7f7f7fu;
                        tc::tmem_st4(tm + lane_base + COL_SFB + (uint32_t)(4 * s), w, 0x7f7f7f7fu, 0x7f7f7f7fu,
                                     0x7f7f7f7fu);
                    }
                }
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(B.b_ready);
                ++nb;
                key = it.key;
            }
            // weight scale factors by groups of K steps [8k, 8k+8) cut to the segment;
            // the previous segment's epilogue runs once two groups are queued
            int ngrp = 0;
            for (int g0 = sg.j0; g0 < sg.j1 && !dead;) {
                const int g1 = min((g0 & ~(GRP - 1)) + GRP, sg.j1);
                const int ga = g0 & ~(GRP - 1);
                uint32_t w[GRP][2][4];
                if (it.shared) {
                    const uint8_t *s8 = (const uint8_t *)(sg.c < 2 ? a.ss13 : a.ss2);
                    const int kb = K / 128;
#pragma unroll
                    for (int jj = 0; jj < GRP; ++jj)
#pragma unroll
                        for (int tt = 0; tt < 2; ++tt) {
                            const int rb = sg.c < 2 ? tt * (I / 128) + it.blk : 2 * it.blk + tt;
                            const uint32_t v = (ga + jj >= g0 && ga + jj < g1)
                                                   ? 0x01010101u * (uint32_t)__ldg(s8 + (size_t)rb * kb + ga + jj)
                                                   : 0x7f7f7f7fu;
                            w[jj][tt][0] = w[jj][tt][1] = w[jj][tt][2] = w[jj][tt][3] = v;
                        }
                } else {
                    const int ks = K / 32;
                    const uint8_t *sb = sg.c < 2 ? a.w13_s + (size_t)it.el * (2 * I) * ks
                                                 : a.w2_s + (size_t)it.el * D * ks;
#pragma unroll
                    for (int tt = 0; tt < 2; ++tt)
#pragma unroll
                        for (int r1 = 0; r1 < 4; ++r1) {
                            const int rr = 32 * r1 + lane;
                            const int grow = sg.c < 2 ? tt * I + it.blk * 128 + rr : it.blk * 256 + tt * 128 + rr;
                            const uint8_t *src = sb + (size_t)grow * ks + (size_t)ga * 4;
                            if ((nst & (GRP - 1)) == 0) {
                                const uint4 lo = ldg128(src), hi = ldg128(src + 16);
                                w[0][tt][r1] = lo.x; w[1][tt][r1] = lo.y; w[2][tt][r1] = lo.z; w[3][tt][r1] = lo.w;
                                w[4][tt][r1] = hi.x; w[5][tt][r1] = hi.y; w[6][tt][r1] = hi.z; w[7][tt][r1] = hi.w;
                            } else {
#pragma unroll
                                for (int jj = 0; jj < GRP; ++jj)
                                    w[jj][tt][r1] = (ga + jj >= g0 && ga + jj < g1)
                                                        ? __ldg(reinterpret_cast<const uint32_t *>(src) + jj)
                                                        : 0x7f7f7f7fu;
                            }
                        }
                }
                if (gi >= 2 && !wwait(B.sfa_free + (gi & 1), ((gi >> 1) - 1) & 1)) break;
                tc::fence_after_sync();
                const uint32_t cbase = tm + lane_base + COL_SFA + (uint32_t)((gi & 1) * (GRP * 8));
#pragma unroll
                for (int jj = 0; jj < GRP; ++jj)
                    if (ga + jj >= g0 && ga + jj < g1) {
#pragma unroll
                        for (int tt = 0; tt < 2; ++tt)
                            tc::tmem_st4(cbase + (uint32_t)((jj * 2 + tt) * 4), w[jj][tt][0], w[jj][tt][1],
                                         w[jj][tt][2], w[jj][tt][3]);
                    }
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(B.sfa_ready + (gi & 1));
                ++gi;
                ++ngrp;
                g0 = g1;
                if (have_prev && (ngrp == 2 || (ngrp == 1 && g1 == sg.j1))) {
                    epilogue(prev);
                    have_prev = false;
                }
            }
            if (dead) break;
            prev = sg;
            have_prev = true;
        }
        if (have_prev && !dead) epilogue(prev);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == W_PROD) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tm, 512);
    }
}

// The owner's rows after expert parallelism over peer memory: wait (bounded) for
// every rank's combine epoch, then y[t] = bf16(sum over ranks, in rank order, of
// the partial rows the ranks wrote to this rank's receive buffer).
__global__ void k_ep_finish(unsigned *flags, const float *yrecv, int P, int Tr, int D, __nv_bfloat16 *y,
                            int *err, long long limit) {
    __shared__ int ok;
    const unsigned epoch = __ldcg(flags + EP_CTR) + 1u;
    if (threadIdx.x == 0) {
        bool good = true;
        for (int p = 0; p < P && good; ++p)
            good = spin_until(flags + EP_MAX_RANKS + p, epoch, err, limit, ld_acquire_sys_u32);
        ok = good;
    }
    __syncthreads();
    if (!ok) return;
    const long long n = (long long)Tr * D;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        float acc = __ldcg(yrecv + i);
        for (int p = 1; p < P; ++p) acc += __ldcg(yrecv + (long long)p * n + i);
        y[i] = __float2bfloat16_rn(acc);
    }
    // the last block advances this rank's epoch counter (every block has read it)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(flags + EP_FIN, 1u) == gridDim.x - 1) {
            flags[EP_FIN] = 0u;
            __threadfence();
            flags[EP_CTR] = epoch;
        }
    }
}

}  // namespace fus
