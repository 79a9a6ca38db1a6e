// wf_moe_tc.cuh - the expert phases of the MoE layer on the 5th-generation
// tensor cores (tcgen05), included by wf_moe.cu inside namespace wf.
//
//   phase 2 (w1/w3): h = act_quant(weights * silu(x W1^T) * (x W3^T))  per expert
//   phase 3 (w2):    o = h W2^T per expert, then the ascending-expert combine
//
// reference: Expert.forward (architecture.py:728-741) on fp4_gemm / fp8_gemm
// (torch_ops.py:93-108), MoE.forward's combine (architecture.py:785-794).
//
// Work list.  An item is one token group (<= 16 tokens of one expert, or of
// the shared expert) times one weight row block: for phase 2 the 128 gate rows
// and the matching 128 up rows (one h quantization block), for phase 3 256
// output rows.  Shared-expert items come first, then the routed items in
// ascending local expert order (tables written by the router kernel).  Every
// item has the same number of 128-wide K steps, and the grid splits the
// concatenated K steps of all items evenly (stream-K): a CTA owns the
// contiguous range [S*b/G, S*(b+1)/G).  An item cut by a range boundary
// leaves fp32 partials in per-CTA slots; the last of its segments to finish
// (arrival counter) sums them in segment order, so the result does not depend
// on timing.
//
// One K step = one 32 KB shared-memory stage: 256 weight rows x 128 K, one
// byte per element (FP4 E2M1 is unpacked by TMA type 16U4_ALIGN16B, FP8 E4M3
// is copied as is), 128-byte swizzle, as two M = 128 tiles.
//
// Warp roles (256 threads):
//   warps 0-3  workers: B operand (the item's tokens as E4M3, all K steps) in
//              shared memory, B scales and weight scales in TMEM, epilogue
//              (TMEM -> registers, SwiGLU + quantization or bf16 output)
//   warp 4     TMA producer of the weight stages
//   warps 5-7  MMA issuers: issuer i issues steps i, i+3, i+6, ... of a segment
//              into its own accumulators (one thread issues a block-scaled MMA
//              in ~150 cycles; three keep up with HBM)
#pragma once

namespace mtc {

constexpr int W_PROD = 4, W_ISS0 = 5, NISS = 3;
constexpr int THREADS = 8 * 32;
constexpr int NWK = 128;                 // worker threads
constexpr int MAX_STAGES = 6;            // stage barriers provided
constexpr int STAGE_BYTES = 32768;
constexpr int TILE_BYTES = 16384;
constexpr int NT = 16;                   // tokens per item (MMA N)
constexpr int BSTEP = NT * 128;          // B bytes per K step
constexpr int MAX_STEPS = 32;            // K <= 4096
constexpr int GRP = 8;                   // K steps per weight-scale group
// Stream-K takes at least this many K steps per CTA: with little work (the
// shared expert alone, a few tokens) a finer split only adds partial-sum
// fix-ups to the end of the kernel, which cost more than the streaming they save.
constexpr int MIN_SEG = 16;
// The weight stages and the B operand share one region: B takes nst x BSTEP
// (all K steps of a token group), the stages the rest (4 at K = 4096, 5 at 2048).
constexpr int OFF_A = 0;
constexpr int AB_BYTES = 4 * STAGE_BYTES + MAX_STEPS * BSTEP;  // stages, then B (192 KB)
constexpr int OFF_BAR = OFF_A + AB_BYTES;
constexpr int NBAR = 2 * MAX_STAGES + 10 + NISS;  // ..., fin[NISS]
constexpr int OFF_MISC = (OFF_BAR + NBAR * 8 + 127) / 128 * 128;
constexpr int AM_LD = NT + 4;                    // amax tile row: 16-byte aligned, conflict-free reads
constexpr int OFF_EX = OFF_MISC + 128;           // [128 rows][AM_LD] |h|, then [NT] scales
constexpr int EX_BYTES = (128 * AM_LD + 2 * NT) * 4;
constexpr int OFF_ROUTE = OFF_EX + EX_BYTES;     // act_expert, act_off, act_it
constexpr int ROUTE_BYTES = 3 * (MAX_E + 1) * 4;
constexpr int OFF_TOK = OFF_ROUTE + ROUTE_BYTES;  // w2 phase: tok_pairs (int16), then tok_np (uint8)
constexpr int TOK_BYTES = MAX_T * MAX_K * 2 + MAX_T;
constexpr int SMEM = OFF_TOK + TOK_BYTES + 1024;  // + alignment slack
static_assert(MAX_PAIRS <= 32767, "pair indices fit int16");
static_assert(SMEM <= 232448, "shared memory budget");
static_assert(OFF_EX % 16 == 0 && (AM_LD * 4) % 16 == 0, "float4 rows of the amax tile");
static_assert(2 * MAX_T * MAX_K * 2 <= EX_BYTES, "the w2 phase stages per-slot routing in the amax tile");
// TMEM columns (512 allocated)
constexpr uint32_t COL_D = 0;      // [issuer][buf][tile] x NT
constexpr uint32_t COL_SFB = 192;  // [K step] x 4
constexpr uint32_t COL_SFA = 320;  // [group buf][step in group][tile] x 4
static_assert(COL_D + NISS * 2 * 2 * NT <= COL_SFB, "accumulator columns");
static_assert(COL_SFB + MAX_STEPS * 4 <= COL_SFA, "B scale columns");
static_assert(COL_SFA + 2 * GRP * 2 * 4 <= 512, "weight scale columns");

struct TcArgs {
    CUtensorMap m_r13;  // routed w1/w3, FP4, 3D {D, I, 2E}: box 128 x 128 x 2 (gate, up)
    CUtensorMap m_s13;  // shared w1/w3, FP8, 3D {D, I, 2}: box 128 x 128 x 2
    CUtensorMap m_r2;   // routed w2, FP4, 2D {I, E*D}: box 128 x 256
    CUtensorMap m_s2;   // shared w2, FP8, 2D {I, D}: box 128 x 256
    const uint8_t *xq, *xs;    // tokens E4M3 [T, D], e8m0 [T, D/128] (router kernel)
    uint8_t *hq, *hqs;         // routed hidden E4M3 [P, I], e8m0 [P, I/128]
    uint8_t *sq, *sqs;         // shared hidden E4M3 [T, I], e8m0 [T, I/128]
    float *part;               // [2 * grid][2][NT/4][128][4] partial slots (float4 per row and 4 tokens)
    unsigned *cnt;             // [items] segment arrivals
};

struct Bars {
    uint64_t *full, *empty, *b_ready, *b_free, *sfa_ready, *sfa_free, *d_ready, *d_free, *fin;
};

__device__ __forceinline__ Bars bars_at(uint8_t *base) {
    uint64_t *b = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    Bars r;
    r.full = b;
    r.empty = b + MAX_STAGES;
    r.b_ready = b + 2 * MAX_STAGES;
    r.b_free = b + 2 * MAX_STAGES + 1;
    r.sfa_ready = b + 2 * MAX_STAGES + 2;  // [2]
    r.sfa_free = b + 2 * MAX_STAGES + 4;   // [2]
    r.d_ready = b + 2 * MAX_STAGES + 6;    // [2]
    r.d_free = b + 2 * MAX_STAGES + 8;     // [2]
    r.fin = b + 2 * MAX_STAGES + 10;       // [NISS] issuer drain
    return r;
}

// Item of phase PH (2: w1/w3, 3: w2).
struct TItem {
    int shared, el, blk, tok0, ntok, key;
};

struct TRoute {
    const int *act_expert, *act_off, *act_it;
    int n_act, ns, nblk;
};

// Walks items in increasing order (each role keeps its own).
struct TCursor {
    int ai = 0;
    bool init = false;
};

template <int PH>
__device__ __forceinline__ TItem decode(const MoeArgs &a, const TRoute &r, TCursor &c, int i) {
    TItem it;
    if (i < r.ns) {
        const int tg = i / r.nblk;
        it.shared = 1; it.el = 0; it.blk = i - tg * r.nblk;
        it.tok0 = a.sh0 + tg * NT; it.ntok = min(NT, a.shT - tg * NT);
    } else {
        const int j = i - r.ns;
        if (!c.init) {
            int lo = 0, hi = r.n_act - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (r.act_it[mid] <= j) lo = mid; else hi = mid - 1;
            }
            c.ai = lo;
            c.init = true;
        }
        while (c.ai + 1 < r.n_act && j >= r.act_it[c.ai + 1]) ++c.ai;
        const int local = j - r.act_it[c.ai];
        const int tg = local / r.nblk;
        const int p0 = r.act_off[c.ai], ta = r.act_off[c.ai + 1] - p0;
        it.shared = 0; it.el = r.act_expert[c.ai] - a.e0; it.blk = local - tg * r.nblk;
        it.tok0 = p0 + tg * NT; it.ntok = min(NT, ta - tg * NT);
    }
    it.key = i / r.nblk;
    return it;
}

// CTA owning K step x of the S steps split over G CTAs
__device__ __forceinline__ int cta_of(long long x, long long S, int G) {
    return (int)(((x + 1) * G - 1) / S);
}
__device__ __forceinline__ long long cta_start(int b, long long S, int G) { return S * b / G; }

// Wait on another role's progress (bounded by the launch's limit); a timeout stops every role.
__device__ __forceinline__ bool twait(uint64_t *bar, uint32_t parity, int *err, volatile int *abort,
                                      long long limit) {
    if (*abort) return false;
    if (!wf_wait(bar, parity, err, limit)) { *abort = 1; return false; }
    return true;
}

// OR of `v` over the `n` threads of named barrier `id` (every one of them must call it)
__device__ __forceinline__ int bar_or(int id, int n, int v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(v), "r"(id), "r"(n)
        : "memory");
    return r;
}

__device__ __forceinline__ uint8_t e4m3_byte(float v) {
    return (uint8_t)(f32x2_to_e4m3x2(v, 0.f) & 0xffu);
}

// Segment of one CTA's range: item i, K steps [j0, j1), its ordinal q.
struct Seg {
    int i, j0, j1, q;
};

template <int PH>
__global__ void __launch_bounds__(THREADS, 1) k_moe_tc(const __grid_constant__ MoeArgs a,
                                                       const __grid_constant__ TcArgs t) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Bars B = bars_at(base);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(base + OFF_MISC);
    volatile int *abort = reinterpret_cast<volatile int *>(base + OFF_MISC) + 1;
    volatile int *flag = reinterpret_cast<volatile int *>(base + OFF_MISC) + 2;
    float *ex = reinterpret_cast<float *>(base + OFF_EX);
    int *rt_s = reinterpret_cast<int *>(base + OFF_ROUTE);
    int16_t *tp_s = reinterpret_cast<int16_t *>(base + OFF_TOK);
    uint8_t *np_s = base + OFF_TOK + MAX_T * MAX_K * 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        // empty: every issuer releases every stage use (see the issuer loop)
        for (int s = 0; s < MAX_STAGES; ++s) { mbar_init(B.full + s, 1); mbar_init(B.empty + s, NISS); }
        mbar_init(B.b_ready, 4);
        mbar_init(B.b_free, NISS);
        for (int j = 0; j < 2; ++j) {
            mbar_init(B.sfa_ready + j, 4); mbar_init(B.sfa_free + j, NISS);
            mbar_init(B.d_ready + j, NISS); mbar_init(B.d_free + j, 4);
        }
        for (int j = 0; j < NISS; ++j) mbar_init(B.fin + j, 1);
        *abort = 0;
        *flag = 0;
        fence_mbar_init();
    }
    if (warp == W_PROD) { tc::tmem_alloc(tmem_slot, 512); tc::tmem_relinquish(); }
    // The w1/w3 phase reads the router kernel's tables: everything waits for it.
    // The w2 phase reads the same tables, and the router kernel completed before
    // the w1/w3 kernel passed its own wait (which precedes its launch of this
    // one), so they are read here at once, through L2; the producer then fills
    // the weight ring while the w1/w3 kernel finishes.  Only the worker warps,
    // which read its outputs (h, the shared hidden rows, their scales), wait.
    if (PH == 2) {
        pdl_wait();
        pdl_launch_dependents();
    }
    // the header and every table entry the workspace holds, in one round trip
    // (entries past n_act are never used)
    const int n_act = __ldcg(a.hdr + H_NACT);
    const int n_rt = __ldcg(a.hdr + (PH == 2 ? H_IT2 : H_IT3));
    TRoute r;
    {
        const int *src_it = PH == 2 ? a.act_it2 : a.act_it3;
        for (int k = threadIdx.x; k <= a.El; k += THREADS) {
            const int ve = __ldcg(a.act_expert + k), vo = __ldcg(a.act_off + k), vi = __ldcg(src_it + k);
            rt_s[k] = ve;
            rt_s[(MAX_E + 1) + k] = vo;
            rt_s[2 * (MAX_E + 1) + k] = vi;
        }
        r.act_expert = rt_s;
        r.act_off = rt_s + (MAX_E + 1);
        r.act_it = rt_s + 2 * (MAX_E + 1);
        r.n_act = n_act;
        r.nblk = PH == 2 ? a.I / 128 : a.D / 256;
        r.ns = r.nblk * cdiv(a.shT, NT);  // shared items
        if (PH == 3) {
            // The combine's lists: each token's pairs in ascending expert order
            // (a token's kept experts are distinct, so a slot's place is the number
            // of its kept slots with a smaller expert), from the router kernel's
            // per-slot expert (a.ridx) and pair (a.tok_pairs, -1: none), staged in
            // the amax tile, which this phase does not use.
            const int TK = a.T * a.topk, K = a.topk;
            int16_t *sr = reinterpret_cast<int16_t *>(ex);
            int16_t *sp = sr + MAX_T * MAX_K;
            for (int k = threadIdx.x; k < TK; k += THREADS) {
                const int e = __ldcg(a.ridx + k), pr = __ldcg(a.tok_pairs + k);
                sr[k] = (int16_t)e;
                sp[k] = (int16_t)pr;
            }
            __syncthreads();
            for (int t = threadIdx.x; t < a.T; t += THREADS) {
                int n = 0;
                for (int j = 0; j < K; ++j) {
                    const int pr = sp[t * K + j];
                    if (pr < 0) continue;
                    const int e = sr[t * K + j];
                    int rank = 0;
                    for (int j2 = 0; j2 < K; ++j2) rank += (sp[t * K + j2] >= 0 && sr[t * K + j2] < e) ? 1 : 0;
                    tp_s[t * K + rank] = (int16_t)pr;
                    ++n;
                }
                np_s[t] = (uint8_t)n;
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tm = *tmem_slot;

    const int D = a.D, I = a.I;
    const int K = PH == 2 ? D : I;
    const int nst = K / 128;
    // stages: what the B operand leaves of the shared region
    const int nstg = min(MAX_STAGES, (AB_BYTES - nst * BSTEP) / STAGE_BYTES);
    uint8_t *const Bbase = base + OFF_A + nstg * STAGE_BYTES;
    const int n_items = r.ns + n_rt;
    const long long S = (long long)n_items * nst;
    // the CTAs that share the S steps (the others have none)
    const int G = (int)max(1LL, min((long long)gridDim.x, S / MIN_SEG));
    const long long u0 = min(S, cta_start(blockIdx.x, S, G)), u1 = min(S, cta_start(blockIdx.x + 1, S, G));
    if (PH == 3 && n_items == 0 && warp < 4) {
        // no item at all (a routed-only call whose shard got no tokens): the combine
        // still writes every row block (zeros)
        pdl_wait();
        pdl_launch_dependents();
        for (int rb = blockIdx.x; rb < D / 256; rb += gridDim.x) combine_rows_v8<NWK>(a, rb * 256, 256, np_s, tp_s);
    }
    // segment after `sg` (or the first one when sg.q < 0); false at the end of the range
    auto next_seg = [&](Seg &sg) -> bool {
        const long long u = sg.q < 0 ? u0 : (long long)sg.i * nst + sg.j1;
        if (u >= u1) return false;
        sg.i = (int)(u / nst);
        sg.j0 = (int)(u - (long long)sg.i * nst);
        sg.j1 = (int)min((long long)nst, sg.j0 + (u1 - u));
        sg.q += 1;
        return true;
    };

    if (warp == W_PROD) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = tc::policy_evict_first();
            TCursor cur;
            Seg sg{0, 0, 0, -1};
            int gs = 0, st = 0, lap = 0;  // step count; its stage and ring lap
            while (!*abort && next_seg(sg)) {
                const TItem it = decode<PH>(a, r, cur, sg.i);
                const uint32_t tx = it.shared ? STAGE_BYTES : STAGE_BYTES / 2;
                for (int j = sg.j0; j < sg.j1; ++j, ++gs, lap += (st + 1 == nstg), st = (st + 1 == nstg) ? 0 : st + 1) {
                    if (gs >= nstg && !twait(B.empty + st, (lap - 1) & 1, a.err, abort, a.wait_limit)) break;
                    uint8_t *dst = base + OFF_A + st * STAGE_BYTES;
                    mbar_arrive_expect_tx(B.full + st, tx);
                    if (PH == 2) {
                        if (it.shared) tc::tma_load_3d_hint(dst, &t.m_s13, j * 128, it.blk * 128, 0, B.full + st, pol);
                        else tc::tma_load_3d_hint(dst, &t.m_r13, j * 128, it.blk * 128, 2 * it.el, B.full + st, pol);
                    } else {
                        if (it.shared) tc::tma_load_2d_hint(dst, &t.m_s2, j * 128, it.blk * 256, B.full + st, pol);
                        else tc::tma_load_2d_hint(dst, &t.m_r2, j * 128, it.el * D + it.blk * 256, B.full + st, pol);
                    }
                }
            }
            // every issued copy lands before the CTA may exit
            for (int k = 0; k < nstg && k < gs; ++k) {
                const int g = gs - 1 - k;
                wf_wait(B.full + g % nstg, (g / nstg) & 1, a.err);
            }
        }
    } else if (warp >= W_ISS0) {
        // ------------------------------------------------------------ MMA issuers
        const int ii = warp - W_ISS0;
        if (lane == 0) {
            TCursor cur;
            Seg sg{0, 0, 0, -1};
            int gs = 0, gi = 0, nb = 0, key = -1;
            int st = 0, lap = 0;  // stage and ring lap of step gs
            const uint64_t a0 = tc::smem_desc_sw128(base + OFF_A);
            const uint64_t b0 = tc::smem_desc_sw128(Bbase);
            bool more = next_seg(sg);
            while (more && !*abort) {
                const TItem it = decode<PH>(a, r, cur, sg.i);
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
                bool first = true;
                bool ok = true;
                int own = 0;  // issuer of step j: (j - j0) mod NISS
                for (int j = sg.j0; j < sg.j1; ++j, ++gs, own = (own + 1 == NISS) ? 0 : own + 1,
                                                lap += (st + 1 == nstg), st = (st + 1 == nstg) ? 0 : st + 1) {
                    // weight-scale groups: K steps [8k, 8k+8) of the item, cut to the segment
                    const int gj = j & (GRP - 1);
                    if (j == sg.j0 || gj == 0) {
                        if (!twait(B.sfa_ready + (gi & 1), (gi >> 1) & 1, a.err, abort, a.wait_limit)) { ok = false; break; }
                    }
                    // Every issuer waits for every stage use, not only its own: a parity
                    // wait is valid only while the barrier is at most one phase away,
                    // and an issuer that skipped the previous use of this stage could
                    // otherwise see its still-pending phase as this one's.  Non-owners
                    // release the use at once; the producer refills a stage when all
                    // issuers have passed it and the owner's MMAs are done.
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
                more = next_seg(sg);
                // the B operand may be replaced once this token set's MMAs are done
                if (!more || (sg.i / r.nblk) != key_now) tc::commit(B.b_free);
            }
            // all of this thread's MMAs complete before TMEM is released
            tc::commit(B.fin + ii);
            wf_wait(B.fin + ii, 0, a.err);
        }
    } else {
        // ------------------------------------------------------------ workers
        const int wq = warp;  // TMEM lane quadrant
        const int tid = threadIdx.x;
        const uint32_t lane_base = (uint32_t)(32 * wq) << 16;
        const int row = 32 * wq + lane;  // accumulator lane = row within a 128-row tile
        TCursor cur, cur_e;
        Seg sg{0, 0, 0, -1};
        int gi = 0, nb = 0, key = -1;
        uint8_t *Bsm = Bbase;
        // The four worker warps share named barriers, so each wait ends in one
        // decision for all of them: a timeout seen by any warp stops every warp.
        bool dead = false;
        auto wwait = [&](uint64_t *bar, uint32_t parity) -> bool {
            const bool ok = twait(bar, parity, a.err, abort, a.wait_limit);
            if (bar_or(1, NWK, !ok)) dead = true;
            return !dead;
        };

        auto epilogue = [&](const Seg &e) {
            const TItem it = decode<PH>(a, r, cur_e, e.i);
            const int buf = e.q & 1;
            if (!wwait(B.d_ready + buf, (e.q >> 1) & 1)) return;
            tc::fence_after_sync();
            // sum of the issuers' accumulators in issuer order (issuer i has steps
            // iff the segment has more than i)
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
                // stream-K: this segment's partial sums go to the CTA's slot; the last
                // segment of the item to arrive sums all of them in segment order
                const long long is = (long long)e.i * nst;
                const int mine = blockIdx.x * 2 + (u0 >= is ? 0 : 1);
                // slot layout [gate/up][token/4][row][4]: each warp access is 512
                // contiguous bytes, written here and read back by the fix-up
                float4 *ps = reinterpret_cast<float4 *>(t.part + (size_t)mine * (2 * 128 * NT));
#pragma unroll
                for (int c = 0; c < NT / 4; ++c) {
                    if (4 * c >= ntok) break;
                    ps[c * 128 + row] = make_float4(g[4 * c], g[4 * c + 1], g[4 * c + 2], g[4 * c + 3]);
                    ps[(NT / 4 + c) * 128 + row] = make_float4(u[4 * c], u[4 * c + 1], u[4 * c + 2], u[4 * c + 3]);
                }
                __threadfence();
                bar_sync(1, NWK);
                if (tid == 0) {
                    const int blo = cta_of(is, S, G), bhi = cta_of(is + nst - 1, S, G);
                    int nseg = 0;
                    for (int b = blo; b <= bhi; ++b)
                        nseg += cta_start(b + 1, S, G) > cta_start(b, S, G);
                    const unsigned old = atomicAdd(t.cnt + e.i, 1u);
                    *flag = old == (unsigned)(nseg - 1);
                }
                bar_sync(1, NWK);
                const int last = *flag;
                bar_sync(1, NWK);
                if (!last) return;
                __threadfence();
#pragma unroll
                for (int n = 0; n < NT; ++n) { g[n] = 0.f; u[n] = 0.f; }
                const int blo = cta_of(is, S, G), bhi = cta_of(is + nst - 1, S, G);
#pragma unroll 2
                for (int b = blo; b <= bhi; ++b) {
                    const long long ub = cta_start(b, S, G);
                    if (cta_start(b + 1, S, G) <= ub) continue;
                    const float4 *pp =
                        reinterpret_cast<const float4 *>(t.part + (size_t)(b * 2 + (ub >= is ? 0 : 1)) * (2 * 128 * NT));
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
                if (tid == 0) t.cnt[e.i] = 0u;
            }
            if (PH == 2) {
                // SwiGLU (architecture.py:733-741) then act_quant of this 128-row block.
                // The per-token amax over the 128 rows goes through a shared-memory
                // transpose: |h| tile [row][token], 8 threads per token reduce it.
                float h[NT];
#pragma unroll
                for (int c = 0; c < NT / 4; ++c) {
                    if (4 * c >= ntok) break;  // whole chunks of 4 tokens
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int n = 4 * c + k;
                        float hv = swiglu(g[n], u[n], a.swiglu_limit);
                        if (!it.shared) hv = (n < ntok ? __ldg(a.pair_w + it.tok0 + n) : 0.f) * hv;
                        h[n] = n < ntok ? bf16r(hv) : 0.f;
                    }
                    *reinterpret_cast<float4 *>(ex + row * AM_LD + 4 * c) =
                        make_float4(fabsf(h[4 * c]), fabsf(h[4 * c + 1]), fabsf(h[4 * c + 2]), fabsf(h[4 * c + 3]));
                }
                bar_sync(1, NWK);
                float *inv_s = ex + 128 * AM_LD;        // [NT] 1/scale
                uint32_t *sb_s = reinterpret_cast<uint32_t *>(inv_s + NT);  // [NT] e8m0 byte
                {
                    const int n = tid >> 3, part = tid & 7;  // 16 tokens x 8 threads
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
                    const size_t prow = (size_t)(it.tok0 + n);
                    dq[prow * I + it.blk * 128 + row] = e4m3_byte(qv);
                }
                if (tid < ntok) ds[(size_t)(it.tok0 + tid) * ib + it.blk] = (uint8_t)sb_s[tid];
                bar_sync(1, NWK);  // the tile is reused by the next epilogue
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
                    const unsigned target =
                        (unsigned)(a.hdr[H_TGT] + cdiv(a.shT, NT));
                    const unsigned old = atomicAdd(a.cnt_rb + it.blk, 1u);
                    *flag = old == target - 1;
                }
                bar_sync(1, NWK);
                const int last = *flag;
                bar_sync(1, NWK);
                if (last) {
                    __threadfence();
                    combine_rows_v8<NWK>(a, it.blk * 256, 256, np_s, tp_s);
                    if (tid == 0) a.cnt_rb[it.blk] = 0u;
                }
            }
        };

        // Weight scale factors of K steps [g0, end of g0's aligned group of GRP, cut
        // at j1) of item `it` into TMEM slot gi & 1 for the issuers; returns the
        // group's end, or -1 when a wait ran out.  They depend on the weights only.
        auto sfa_group = [&](const TItem &it, int g0, int j1) -> int {
            const int g1 = min((g0 & ~(GRP - 1)) + GRP, j1);
            const int ga = g0 & ~(GRP - 1);  // first step of the aligned group
            // global loads first; the wait below only guards the TMEM slot
            uint32_t w[GRP][2][4];
            if (it.shared) {
                const uint8_t *s8 = (const uint8_t *)(PH == 2 ? a.ss13 : a.ss2);
                const int kb = K / 128;
#pragma unroll
                for (int jj = 0; jj < GRP; ++jj)
#pragma unroll
                    for (int tt = 0; tt < 2; ++tt) {
                        const int rb = PH == 2 ? tt * (I / 128) + it.blk : 2 * it.blk + tt;
                        const uint32_t v = (ga + jj >= g0 && ga + jj < g1)
                                               ? 0x01010101u * (uint32_t)__ldg(s8 + (size_t)rb * kb + ga + jj)
                                               : 0x7f7f7f7fu;
                        w[jj][tt][0] = w[jj][tt][1] = w[jj][tt][2] = w[jj][tt][3] = v;
                    }
            } else {
                const int ks = K / 32;
                const uint8_t *sb = PH == 2 ? a.w13_s + (size_t)it.el * (2 * I) * ks
                                            : a.w2_s + (size_t)it.el * D * ks;
#pragma unroll
                for (int tt = 0; tt < 2; ++tt)
#pragma unroll
                    for (int r1 = 0; r1 < 4; ++r1) {
                        const int rr = 32 * r1 + lane;
                        const int grow = PH == 2 ? tt * I + it.blk * 128 + rr : it.blk * 256 + tt * 128 + rr;
                        const uint8_t *src = sb + (size_t)grow * ks + (size_t)ga * 4;
                        if ((nst & (GRP - 1)) == 0) {
                            // the row's 8 words of this group: two 16-byte loads
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
            if (gi >= 2 && !wwait(B.sfa_free + (gi & 1), ((gi >> 1) - 1) & 1)) return -1;
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
            return g1;
        };
        // The w2 phase stages the first group of the CTA's first segment before the
        // wait for the w1/w3 kernel, whose outputs its B operand is: the first MMA
        // then starts as soon as B is in place.  The w1/w3 phase cannot start before
        // its wait (the item comes from the routing); it sends the group's scale
        // rows towards L2 and loads B, whose latency the prefetch then hides.
        int g_pre = -1;
        {
            Seg s0{0, 0, 0, -1};
            TCursor c0;
            if (next_seg(s0)) {
                const TItem it0 = decode<PH>(a, r, c0, s0.i);
                if (PH == 3) {
                    g_pre = sfa_group(it0, s0.j0, s0.j1);
                } else if (!it0.shared) {
                    const int ks = K / 32, ga = s0.j0 & ~(GRP - 1);
                    const uint8_t *sb = a.w13_s + (size_t)it0.el * (2 * I) * ks;
#pragma unroll
                    for (int tt = 0; tt < 2; ++tt)
#pragma unroll
                        for (int r1 = 0; r1 < 4; ++r1) {
                            const int grow = tt * I + it0.blk * 128 + 32 * r1 + lane;
                            asm volatile("prefetch.global.L2 [%0];" ::"l"(sb + (size_t)grow * ks + (size_t)ga * 4));
                        }
                }
            }
        }
        if (PH == 3) {
            pdl_wait();
            pdl_launch_dependents();
        }

        Seg prev{0, 0, 0, -1};
        bool have_prev = false;
        while (!dead && next_seg(sg)) {
            const TItem it = decode<PH>(a, r, cur, sg.i);
            if (it.key != key) {
                // new token set: E4M3 rows of all K steps, swizzled, and their scales
                if (nb > 0 && !wwait(B.b_free, (nb - 1) & 1)) break;
                const uint8_t *src0;
                const uint8_t *sc0;
                size_t rstride, sstride;
                if (PH == 2) { src0 = t.xq; sc0 = t.xs; rstride = D; sstride = D / 128; }
                else if (it.shared) { src0 = t.sq; sc0 = t.sqs; rstride = I; sstride = I / 128; }
                else { src0 = t.hq; sc0 = t.hqs; rstride = I; sstride = I / 128; }
                auto tok_row = [&](int n) -> size_t {
                    if (PH == 2 && !it.shared) return (size_t)__ldg(a.pair_tok + it.tok0 + n);
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
                            v[k] = ldg128(src0 + tok_row(n) * rstride + s * 128 + ch * 16);
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
                        const uint32_t w = tv ? 0x01010101u * (uint32_t)__ldg(sr + s) : 0x7f7f7f7fu;
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
            // the previous segment's epilogue runs once two groups are queued (the
            // first segment's first group went ahead of its B operand)
            int ngrp = 0;
            for (int g0 = (sg.q == 0 && g_pre > 0) ? g_pre : sg.j0; g0 < sg.j1 && !dead;) {
                const int g1 = sfa_group(it, g0, sg.j1);
                if (g1 < 0) break;
                ++ngrp;
                g0 = g1;
                if (have_prev && (ngrp == 2 || (ngrp == 1 && g1 == sg.j1))) epilogue(prev);
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

}  // namespace mtc
