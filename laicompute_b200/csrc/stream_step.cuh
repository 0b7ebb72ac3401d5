// The decode step of one sequence as one persistent kernel that never stops
// streaming weights (the batch-1 latency path of LlamaRuntime::step, reference
// src/inference_v2.cpp:31, for Q4_0 or Q8_0 projections with an FP16 KV cache).
//
// One CTA per SM; inside a CTA sixteen consumer warps, one producer warp and two
// epilogue warps.
//
//  * Each consumer warp streams its own contiguous share of the CTA's tile-blocks
//    of every projection phase, in step order, through its own ring of three
//    ~2.2 KB shared-memory stages (1-D bulk copies, cp.async.bulk + mbarrier,
//    issued by its lane 0). Weights never depend on the step's activations, so a
//    warp's ring keeps filling with the next phase's bytes while the warp waits
//    for the other SMs at a phase boundary, and HBM stays busy across the
//    boundaries that separate kernel launches elsewhere.
//  * The producer warp copies the attention phases' K and V chunks (the rows of
//    earlier steps) into a shared ring of 9 KB stages, its lanes issuing a batch
//    of stages together.
//  * The consumers run the phases in order. Before a phase they wait until every
//    CTA has arrived at the previous phase's counter (a bounded spin on a 64-bit
//    monotonic counter: target = CTAs x launch epoch), copy the phase's input
//    activation records into shared memory with one bulk copy and, for a
//    projection after an rmsnorm, form 1/rms from the per-tile sums of squares
//    the producing phase wrote.
//  * A consumer warp hands the 16 row sums of each row tile its share touches
//    (a "piece") to the epilogue warps through its own small queue. An epilogue
//    warp adds a tile's pieces in warp order and runs the tile's global epilogue,
//    so consumer warps never wait on a global round trip.
//
// Phases of a step: EMB (token row -> residual x), then per layer QKV (rmsnorm,
// fused [Wq;Wk;Wv], RoPE, K/V append), ATT (GQA attention), O (Wo, residual
// add), GU (rmsnorm, interleaved [Wgate;Wup], SwiGLU), DN (Wdown, residual
// add), and LM (final rmsnorm, lm_head) when the lm_head shares the layers'
// block type.
//
// Projection work is split by whole 16-row tiles: CTA c owns the tiles
// [c T / G, (c+1) T / G) of the phase's T tiles (all their block columns), so a
// tile's row sums never cross CTAs and its epilogue needs no global round trip;
// inside the CTA the tile-blocks are split evenly over the consumer warps.
// Epilogues that feed the next projection also write its activation records, one
// 8-element group at a time.
//
// The matvec inner loop (one sequence) is integer: the activation record of a
// 32-column block holds, per 8-element group, the values scaled by a power of two
// and split into three balanced base-128 int8 digits, plus -8 x (sum of the
// group) for Q4_0's nibble offset and the inverse scale; a lane multiplies a
// row's 8 quants with each digit word by dp4a, joins the three exact integer sums
// and adds d_row x 2^-s x sum in FP32 (ls_block_dp4 below; the team kernel instead
// forms a whole block's sums with one mma.m16n8k32, tile_block_dp in mv_streamk.cuh).
//
// Every wait is bounded (about one second of SM clocks); a wait that runs out
// records its code in `err`, and once `err` is set the dependency waits stop
// waiting, so a failed step still ends. No wait is on a peer GPU.
#pragma once
#include "mma_matvec.cuh"
#include "mv_streamk.cuh"
#include "tiles.cuh"

namespace laic {

constexpr int kLsWarps = 16;                         // consumer warps
constexpr int kLsEpi = 2;                            // epilogue warps
constexpr int kLsThreads = (kLsWarps + 1 + kLsEpi) * 32;  // + the producer warp + the epilogue warps
constexpr int kLsStage = 9216;                       // attention ring stage bytes (a K or V chunk)
constexpr int kLsWRing = 3;                          // weight stages in flight per consumer warp
constexpr int kLsRec = 128;                          // activation record bytes per 32-column block (+ 4 B scale)
constexpr int kLsMaxStages = 24;
constexpr int kLsPQ = 4;                             // tile pieces in flight from one consumer warp to the
                                                     // epilogue warps (a multiple of kLsEpi)
constexpr int kLsIssue = 8;                          // ring stages the producer warp's lanes issue together
constexpr long long kLsSpin = 2000000000LL;          // clock cycles a dependency wait may take
// Trace stamps per CTA and phase: [0] start, [1] inputs ready, [2] warp 0's own work done
// (attention: before the head ticket), [3] every warp's work done (attention: after the
// ticket and any head merge), [4] done (before the arrival).
constexpr int kLsStamps = 5;

// tile-blocks per weight stage of a consumer warp's ring (about 2.2 KB), and its bytes
__host__ __device__ constexpr int ls_sb(int type) { return type == T_Q4_0 ? 8 : 4; }
__host__ __device__ constexpr int ls_wstage(int type) { return ls_sb(type) * (tile_qbytes(type) + kTileSBytes); }
// positions of one K (or V) chunk per ring stage
__host__ __device__ constexpr int ls_cp(int D) { return kLsStage / (D * 2) >= 64 ? 64 : 32; }

struct LsLayer {
    const uint8_t *qkv_q, *qkv_s, *o_q, *o_s, *gu_q, *gu_s, *dn_q, *dn_s;
    const float* attn_norm;
    const float* ffn_norm;
    void* kc;  // this layer's K cache (FP16)
    void* vc;
};

struct LsParams {
    const LsLayer* layers;
    int L;
    int h, F, hq, kv, heads, kv_heads, rope_pairs;
    int gq;                   // query heads per kv head (at most the kernel's GM)
    float eps, sqrt_d;
    // embedding (any of F16 / Q8_0 / Q4_0, fragment-tile layout)
    int emb_type;
    const uint8_t *emb_q, *emb_s;
    int emb_nb, vocab;
    const unsigned* tokens;   // [1]
    const int* slots;         // [1]
    const int* pos;           // [max_seqs]
    unsigned* counts;         // [max_seqs][vocab] history counts
    // lm_head in the kernel (lm_q != nullptr and lm_on)
    const uint8_t *lm_q, *lm_s;
    int lm_rows;
    int lm_on;                // 0: the LM phase does no work (prefill steps, or an lm_head of another type)
    const float* out_norm;
    float* logits;
    // state
    float *x, *q, *attn, *act;
    const float2* rope_cs;
    long long kv_slot_stride;
    int kv_cap;
    uint8_t *rec_x, *rec_attn, *rec_act;  // activation records of the projections' inputs
    float* ss_x;                          // [h / 16] sums of squares of the residual per row tile
    float* apart;                         // attention partials [kv_head][chunk][G (D + 2)]
    int att_maxch;                        // chunks per kv head the scratch holds
    int att_runs;                         // most CTAs one kv head's chunks can be spread over (one per chunk)
    unsigned* head_tick;                  // [kv_heads]
    unsigned long long* done;             // [phases] arrivals (monotonic)
    unsigned long long* epoch;            // launches completed
    int* err;
    int nstages;                          // ring depth
    unsigned long long* trace;            // optional: [CTA][phase][kLsStamps] globaltimer stamps, then
                                          // [CTA][consumer warp][5] wait statistics (see ls_step_kernel)
};

__device__ __forceinline__ unsigned long long ls_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

enum : int { LS_EMB = 0, LS_QKV = 1, LS_ATT = 2, LS_O = 3, LS_GU = 4, LS_DN = 5, LS_LM = 6 };

__host__ __device__ inline int ls_phases(int L) { return 2 + 5 * L; }
__device__ __forceinline__ int ls_kind(int ph, int L) {
    if (ph == 0) return LS_EMB;
    if (ph == 1 + 5 * L) return LS_LM;
    return 1 + (ph - 1) % 5;
}

// One projection phase: the matrix, its shape, and the weight type of its consumer's records.
struct LsMat {
    const uint8_t *q, *s;
    int rows, nb, ntiles;
    long long nblk;
};
__device__ __forceinline__ LsMat ls_mat(const LsParams& p, int kind, int layer) {
    LsMat m{};
    if (kind == LS_LM) {
        m.q = p.lm_q; m.s = p.lm_s; m.rows = p.lm_on ? p.lm_rows : 0; m.nb = p.h / 32;
    } else {
        const LsLayer& ly = p.layers[layer];
        if (kind == LS_QKV) { m.q = ly.qkv_q; m.s = ly.qkv_s; m.rows = p.hq + 2 * p.kv; m.nb = p.h / 32; }
        if (kind == LS_O) { m.q = ly.o_q; m.s = ly.o_s; m.rows = p.h; m.nb = p.hq / 32; }
        if (kind == LS_GU) { m.q = ly.gu_q; m.s = ly.gu_s; m.rows = 2 * p.F; m.nb = p.h / 32; }
        if (kind == LS_DN) { m.q = ly.dn_q; m.s = ly.dn_s; m.rows = p.h; m.nb = p.F / 32; }
    }
    m.ntiles = (m.rows + 15) / 16;
    m.nblk = (long long)m.ntiles * m.nb;
    return m;
}

// Range [ls_lo(c), ls_lo(c + 1)) of n items owned by CTA c of g (never empty while
// n >= g; with fewer items than CTAs the first n CTAs take one each), and the CTA
// owning item i. The CTAs owning the items of any contiguous span are consecutive.
// 32-bit arithmetic: n * g stays below 2^32 for every phase (the host checks).
__device__ __forceinline__ int ls_lo(unsigned n, int c, int g) {
    return (int)(n >= (unsigned)g ? n * (unsigned)c / (unsigned)g : min((unsigned)c, n));
}
__device__ __forceinline__ int ls_owner(unsigned n, unsigned i, int g) {
    return n >= (unsigned)g ? (int)(((i + 1) * (unsigned)g + n - 1) / n) - 1 : (int)i;
}
// The tile-blocks [lo, hi) of a projection phase owned by CTA c: whole row tiles
// [c T / G, (c+1) T / G) of its T tiles, so that no tile's row sums are split across CTAs.
__device__ __forceinline__ void ls_range(const LsMat& m, int c, int G, int& lo, int& hi) {
    lo = ls_lo((unsigned)m.ntiles, c, G) * m.nb;
    hi = ls_lo((unsigned)m.ntiles, c + 1, G) * m.nb;
}
// The consumer warp owning item i of a CTA's n items (n > 0) split as
// [n w / kLsWarps, n (w + 1) / kLsWarps): the last warp whose range starts at or before i.
__device__ __forceinline__ int ls_warp_owner(unsigned n, unsigned i) {
    return (int)(((i + 1) * (unsigned)kLsWarps + n - 1) / n) - 1;
}
// atomic add with acquire-release ordering at GPU scope: the caller's earlier writes (and
// those of its warp, ordered before by __syncwarp) are visible before the count moves,
// and reads after it see every write released by earlier adds
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* a, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* a) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* a) { return *reinterpret_cast<const volatile int*>(a); }

// Bytes of the activation records of a vector of nb blocks (the integer digit records of
// mv_streamk.cuh: per 8-element group the three base-128 digits, -8 sum x and 2^-s).
__host__ __device__ inline size_t ls_rec_bytes(int nb) { return (size_t)nb * kLsRec; }

// Bounded wait for an mbarrier phase that backs off with nanosleep between polls: a hot
// poll (try_wait and the clock read in a tight loop) takes issue slots and the
// conversion pipe from the warps doing the step's work. Returns false after ~1 s (err set),
// or at once when another wait of the step already failed (err already set), so that a
// failed step ends after one timeout rather than one per wait.
__device__ __forceinline__ bool ls_mbar_wait_backoff(uint64_t* bar, uint32_t parity, int* err, unsigned max_ns = 256) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    unsigned ns = 16;
    while (!mbar_try_wait(bar, parity)) {
        __nanosleep(ns);
        ns = ns < max_ns ? ns * 2 : max_ns;
        if (ld_volatile_i32(err) != 0) return false;
        if (clock64() - t0 > kLsSpin) {
            atomicExch(err, kErrMbarrier);
            return false;
        }
    }
    return true;
}

// After a wait gave up (err set), a warp may leave while bulk copies it issued are still in
// flight: it lingers ~20 us first so that they land in this CTA's shared memory.
__device__ __forceinline__ void ls_settle(const int* err) {
    if (ld_volatile_i32(err) != 0)
        for (int i = 0; i < 20; ++i) __nanosleep(1000);
}

// Named barrier of the consumer warps (the producer warp never joins it).
__device__ __forceinline__ void ls_cbar() { named_sync(1, kLsWarps * 32); }

// One 16x32 tile-block of the integer dot products with four rows per lane: lane (u, t)
// of a half warp does the work of the fragment layout's lanes 8u + t and 8u + 4 + t
// (rows 2u, 2u+8, 2u+1, 2u+9; column group t), so a block's activation record reaches 16
// lanes rather than 32 and the shared-memory delivery per block drops from ~1.4 KB to
// ~0.9 KB (the crossbar delivers 128 B per clock; it bounds this loop). acc[] holds the
// four rows in that order; per (row, group) three dp4a chains, their exact sum
// 2^14 s0 + 2^7 s1 + s2 (+ the group's -8 sum x) and one FP32 multiply-add by d x 2^-s.
template <int WT>
__device__ __forceinline__ void ls_block_dp4(uint32_t q, uint32_t sc, uint32_t xrec, int u, int t, float (&acc)[4]) {
    const uint4 xa = lds128(xrec + t * 32), xb = lds128(xrec + t * 32 + 16);
    const int x8 = (int)xb.z;
    const float sinv = __uint_as_float(xb.w);
    const uint2 dp = lds64(sc + u * 8);  // halves of rows (2u, 2u+8) and (2u+1, 2u+9)
    const float2 d0 = __half22float2(*reinterpret_cast<const __half2*>(&dp.x));
    const float2 d1 = __half22float2(*reinterpret_cast<const __half2*>(&dp.y));
    const float dr[4] = {d0.x, d0.y, d1.x, d1.y};
    uint32_t wl[4], wh[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int l = 8 * u + 4 * h + t;  // the layout lane whose rows these are
        if (WT == T_Q4_0) {
            const uint2 w = lds64(q + l * 8);
            wl[2 * h] = w.x & 0x0F0F0F0Fu; wh[2 * h] = (w.x >> 4) & 0x0F0F0F0Fu;
            wl[2 * h + 1] = w.y & 0x0F0F0F0Fu; wh[2 * h + 1] = (w.y >> 4) & 0x0F0F0F0Fu;
        } else {
            const uint4 w = lds128(q + l * 16);
            wl[2 * h] = w.x; wh[2 * h] = w.y; wl[2 * h + 1] = w.z; wh[2 * h + 1] = w.w;
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        int s0, s1, s2;
        if (WT == T_Q4_0) {
            s2 = dp4a_us(wh[r], xb.y, dp4a_us(wl[r], xb.x, x8));
            s1 = dp4a_us(wh[r], xa.w, dp4a_us(wl[r], xa.z, 0));
            s0 = dp4a_us(wh[r], xa.y, dp4a_us(wl[r], xa.x, 0));
        } else {
            s2 = dp4a_ss(wh[r], xb.y, dp4a_ss(wl[r], xb.x, 0));
            s1 = dp4a_ss(wh[r], xa.w, dp4a_ss(wl[r], xa.z, 0));
            s0 = dp4a_ss(wh[r], xa.y, dp4a_ss(wl[r], xa.x, 0));
        }
        const int v = s0 * 16384 + s1 * 128 + s2;
        acc[r] = fmaf((float)v, dr[r] * sinv, acc[r]);
    }
}

// What a tile's epilogue reads from global memory besides its row sums, loaded by the
// epilogue warp before it waits for the tile's pieces (the loads overlap the consumers'
// work): per lane (row tile * 16 + lane) the residual and the next rmsnorm's weight (O,
// DN), or the RoPE factors of the row (QKV).
struct LsTilePre {
    float x, w;
    float2 cs;
};
// Per phase: the layer's pointers an epilogue needs (loaded once per phase).
struct LsEpiPtrs {
    const float* wn;   // O, DN: weights of the next rmsnorm
    __half *kc, *vc;   // QKV: this layer's K and V caches
};
__device__ __forceinline__ LsEpiPtrs ls_epi_ptrs(const LsParams& p, int kind, int layer) {
    LsEpiPtrs e{nullptr, nullptr, nullptr};
    if (kind == LS_QKV) {
        e.kc = reinterpret_cast<__half*>(p.layers[layer].kc);
        e.vc = reinterpret_cast<__half*>(p.layers[layer].vc);
    } else if (kind == LS_O) {
        e.wn = p.layers[layer].ffn_norm;
    } else if (kind == LS_DN) {
        e.wn = layer + 1 < p.L ? p.layers[layer + 1].attn_norm : p.out_norm;
    }
    return e;
}
template <int D>
__device__ __forceinline__ LsTilePre ls_tile_pre(const LsParams& p, int kind, const LsMat& m, const LsEpiPtrs& e, int tile,
                                                 int pos, int lane) {
    LsTilePre t{0.f, 0.f, make_float2(1.f, 0.f)};
    const int r = tile * 16 + lane;
    if (lane >= 16 || r >= m.rows) return t;
    if (kind == LS_O || kind == LS_DN) {
        t.x = __ldcg(p.x + r);
        t.w = e.wn[r];
    } else if (kind == LS_QKV) {
        const int rr = r < p.hq ? r : r - p.hq;
        const int d = rr % D;
        if (r < p.hq + p.kv && d < 2 * p.rope_pairs) t.cs = p.rope_cs[(size_t)pos * p.rope_pairs + (d >> 1)];
    }
    return t;
}

// The epilogue of one finished row tile (an epilogue warp; lanes 0..15 hold the tile's
// 16 row sums in v).
template <int WT, int D>
__device__ __forceinline__ void ls_finish_tile(const LsParams& p, int kind, const LsMat& m, const LsEpiPtrs& e,
                                               const LsTilePre& t, int tile, float v, float inv, bool norm, int pos,
                                               int sl, int lane) {
    if (norm) v *= inv;
    const int r = tile * 16 + lane;  // this lane's row (lanes 0..15)
    const bool live = lane < 16 && r < m.rows;
    if (kind == LS_LM) {
        if (live) p.logits[r] = v;
    } else if (kind == LS_QKV) {
        const float other = __shfl_xor_sync(0xffffffffu, v, 1);
        if (live) {
            int rr = r, region = 0;
            if (rr >= p.hq) { rr -= p.hq; region = 1; if (rr >= p.kv) { rr -= p.kv; region = 2; } }
            const int d = rr % D;
            float o = v;
            if (region < 2 && d < 2 * p.rope_pairs) {
                // adjacent-pair rotation, unfused like the reference
                if ((d & 1) == 0) o = __fsub_rn(__fmul_rn(v, t.cs.x), __fmul_rn(other, t.cs.y));
                else o = __fadd_rn(__fmul_rn(other, t.cs.y), __fmul_rn(v, t.cs.x));
            }
            if (region == 0) {
                p.q[rr] = o;
            } else {
                __half* base = region == 1 ? e.kc : e.vc;
                base[(size_t)sl * p.kv_slot_stride + ((size_t)(rr / D) * p.kv_cap + pos) * D + d] = __float2half_rn(o);
            }
        }
    } else if (kind == LS_GU) {
        // rows 2o (gate) and 2o+1 (up): act[o] = silu(gate) * up
        // outputs tile * 8 + lane / 2 on the even lanes 0..14: one 8-element group of records
        const float up = __shfl_down_sync(0xffffffffu, v, 1);
        const int o = tile * 8 + (lane >> 1);
        const bool on = live && (lane & 1) == 0;
        const float a = on ? (v / (1.f + expf(-v))) * up : 0.f;
        if (on) p.act[o] = a;
        dp_lane_record<WT>(a, 0.f, lane >> 1, on ? (o >> 3) : -1, p.rec_act, 2, 4, 8);
    } else {  // LS_O, LS_DN: residual add, its sum of squares, records for the next rmsnorm
        // rows tile * 16 + lane on lanes 0..15: two 8-element groups of records of x * (next
        // rmsnorm weight), and the tile's sum of x^2
        float xn = 0.f;
        if (live) {
            xn = t.x + v;
            p.x[r] = xn;
        }
        const float sg = dp_lane_record<WT>(live ? xn * t.w : 0.f, xn * xn, lane & 7, live ? (r >> 3) : -1, p.rec_x,
                                            1, 2, 4);
        const float s8 = __shfl_sync(0xffffffffu, sg, 8);
        if (lane == 0) p.ss_x[tile] = sg + s8;
    }
}

// Named barrier of the consumer and epilogue warps: a phase's inputs are ready (the
// epilogue warps read 1/rms), and a phase's work is complete (before the arrival).
__device__ __forceinline__ void ls_sync_all() { named_sync(2, (kLsWarps + kLsEpi) * 32); }

template <int WT, int D, int GM>
__global__ void __launch_bounds__(kLsThreads, 1) ls_step_kernel(const LsParams p) {
    constexpr int QB = tile_qbytes(WT);
    constexpr int SB = ls_sb(WT);
    constexpr int WS = ls_wstage(WT);
    constexpr int CP = ls_cp(D);
    constexpr int E = D / 32;               // head dims per lane
    constexpr int PPW = CP / kLsWarps;      // chunk positions per consumer warp (scores)
    static_assert(WT == T_Q4_0 || WT == T_Q8_0, "Q4_0 or Q8_0 projections");
    static_assert(PPW >= 1, "at least one chunk position per warp");
    static_assert(kLsPQ % kLsEpi == 0, "an epilogue warp sees every kLsPQ-th piece of a consumer warp before the next use");
    extern __shared__ __align__(128) uint8_t smem[];
    const int NST = p.nstages;  // attention ring stages
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int L = p.L, nph = ls_phases(L);

    // ---- shared memory
    uint8_t* ring = smem;                                                   // [NST][kLsStage] K / V chunks
    uint8_t* wring = ring + (size_t)NST * kLsStage;                         // [kLsWarps][kLsWRing][WS] weights
    uint64_t* full = reinterpret_cast<uint64_t*>(wring + (size_t)kLsWarps * kLsWRing * WS);
    uint64_t* empty = full + kLsMaxStages;
    uint64_t* wfull = empty + kLsMaxStages;                                 // [kLsWarps][kLsWRing]
    uint64_t* xbar = wfull + kLsWarps * kLsWRing;
    uint64_t* pfull = xbar + 2;                                 // [kLsWarps][kLsPQ] a warp's tile piece is in
    uint64_t* pfree = pfull + kLsWarps * kLsPQ;                 // [kLsWarps][kLsPQ] an epilogue warp read it
    float* red = reinterpret_cast<float*>(pfree + kLsWarps * kLsPQ);  // [kLsWarps][kLsPQ][16] piece row sums
    float* qs = red + kLsWarps * kLsPQ * 16;                    // [GM][D] merged attention output
    float* wrun = qs + GM * D;                                  // [att_runs][GM] merge weights of the runs
    int* roff = reinterpret_cast<int*>(wrun + p.att_runs * GM);  // [att_runs] scratch offsets of the runs
    int* ictl = reinterpret_cast<int*>((reinterpret_cast<uintptr_t>(roff + p.att_runs) + 15) & ~uintptr_t(15));
    // ictl: [16] broadcast words, then [kLsWarps][5] trace counters
    uint8_t* act = reinterpret_cast<uint8_t*>(ictl + 16 + kLsWarps * 5);  // activation records of the phase (attention:
                                                                // the warps' softmax states of a run)
    act = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(act) + 127) & ~uintptr_t(127));

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kLsWarps);
        }
        for (int s = 0; s < kLsWarps * kLsWRing; ++s) mbar_init(wfull + s, 1);
        mbar_init(xbar, 1);
        for (int q = 0; q < kLsWarps * kLsPQ; ++q) {
            mbar_init(pfull + q, 1);
            mbar_init(pfree + q, 1);
        }
        mbar_fence_init();
    }
    __syncthreads();

    // =====================================================================
    // producer warp: the attention phases' K and V chunks (rows of earlier steps), in order,
    // into the shared ring as it frees up; every lane steps the same sequence and lane l
    // issues stage i0 + l of each batch
    // =====================================================================
    if (warp == kLsWarps) {
        int ph = -1, kind = LS_EMB;
        const LsLayer* aly = nullptr;
        int apos = 0, asl = 0, nch = 1, it = 0, ihi = 0, j = 0, ch = 0, kvs = 0;
        bool waited = false;
        auto next = [&](const uint8_t*& s0, uint32_t& b0) -> bool {
            for (;;) {
                if (kind == LS_ATT && it < ihi) {
                    const int r0 = ch * CP, nrows = max(0, min(r0 + CP, apos) - r0);
                    const size_t off = (size_t)asl * p.kv_slot_stride + ((size_t)j * p.kv_cap + r0) * D;
                    s0 = reinterpret_cast<const uint8_t*>(reinterpret_cast<const __half*>(kvs ? aly->vc : aly->kc) + off);
                    b0 = (uint32_t)(nrows * D * 2);
                    if (++kvs == 2) { kvs = 0; ++it; if (++ch == nch) { ch = 0; ++j; } }
                    return true;
                }
                if (++ph >= nph) return false;
                kind = ls_kind(ph, L);
                if (kind != LS_ATT) continue;
                if (!waited) { pdl_wait(); waited = true; }  // positions come from the previous step
                asl = p.slots[0];
                apos = p.pos[asl];
                nch = (apos + 1 + CP - 1) / CP;
                const unsigned I = (unsigned)p.kv_heads * nch;
                aly = p.layers + (ph - 1) / 5;
                it = ls_lo(I, c, G); ihi = ls_lo(I, c + 1, G);
                j = it / nch; ch = it % nch; kvs = 0;
            }
        };
        bool ok = true;
        for (int i0 = 0;;) {
            const uint8_t* s0 = nullptr;
            uint32_t b0 = 0;
            int cnt = 0;
            // at most one use of each slot per batch: a lane waits for its slot's previous use
            // only, so its parity wait never aliases a phase two uses back
            const int batch = min(kLsIssue, NST);
            for (int l = 0; l < batch; ++l) {
                const uint8_t* t0;
                uint32_t c0;
                if (!next(t0, c0)) break;
                if (lane == l) { s0 = t0; b0 = c0; }
                ++cnt;
            }
            if (cnt == 0) break;
            if (lane < cnt) {
                const int i = i0 + lane, sl = i % NST;
                const uint32_t r = (uint32_t)(i / NST);
                // the consumers released this slot's previous use (first round: free)
                if (ok && r > 0 && !ls_mbar_wait_backoff(empty + sl, (r - 1) & 1u, p.err)) ok = false;
                if (ok && b0 > 0) {
                    mbar_expect_tx(full + sl, b0);
                    bulk_g2s(ring + (size_t)sl * kLsStage, s0, b0, full + sl);
                } else {
                    mbar_arrive(full + sl);  // nothing to copy (or a failed wait): the stage is ready
                }
            }
            __syncwarp();
            i0 += cnt;
        }
        ls_settle(p.err);
        return;
    }

    // =====================================================================
    // epilogue warps: the row tiles' global epilogues, from the consumers' queue
    // =====================================================================
    if (warp > kLsWarps) {
        const int e = warp - kLsWarps - 1;
        // lane w < kLsWarps: pieces consumer warp w queued in earlier phases (both epilogue
        // warps keep the same counts)
        int wbase = 0;
        for (int ph = 0; ph < nph; ++ph) {
            const int kind = ls_kind(ph, L);
            const int layer = kind == LS_EMB ? 0 : kind == LS_LM ? L - 1 : (ph - 1) / 5;
            ls_sync_all();  // the phase's inputs are ready (1/rms, position, slot)
            if (kind != LS_EMB && kind != LS_ATT) {
                const LsMat m = ls_mat(p, kind, layer);
                const bool norm = kind == LS_QKV || kind == LS_GU || kind == LS_LM;
                const int sl = ictl[2], pos = ictl[3];
                const LsEpiPtrs ep = ls_epi_ptrs(p, kind, layer);
                int lo, hi;
                ls_range(m, c, G, lo, hi);
                const unsigned n = (unsigned)(hi - lo);
                // consumer warp `lane`'s share of the phase: its first tile and its piece count
                const int wl = lo + (int)(n * (unsigned)lane / kLsWarps), wh = lo + (int)(n * (unsigned)(lane + 1) / kLsWarps);
                const int wtile = wl / max(m.nb, 1);
                const int wcnt = lane < kLsWarps && wl < wh ? (wh - 1) / m.nb - wl / m.nb + 1 : 0;
                if (lo < hi) {
                    for (int tile = lo / m.nb, tile_i = 0; tile <= (hi - 1) / m.nb; ++tile, ++tile_i) {
                        if ((tile_i % kLsEpi) != e) continue;
                        // the tile's pieces come from consumer warps wf..wt (their pieces in warp
                        // order); with fewer blocks than warps some of them have an empty share
                        // and queue nothing
                        const int wf = ls_warp_owner(n, (unsigned)(max(lo, tile * m.nb) - lo));
                        const int wt = ls_warp_owner(n, (unsigned)(min(hi, (tile + 1) * m.nb) - 1 - lo));
                        const int kme = wbase + tile - wtile;  // (lane w: warp w's piece number for this tile)
                        const LsTilePre tp = ls_tile_pre<D>(p, kind, m, ep, tile, pos, lane);
                        float v = 0.f;
                        for (int w = wf; w <= wt; ++w) {
                            if (__shfl_sync(0xffffffffu, wcnt, w) == 0) continue;
                            const int k = __shfl_sync(0xffffffffu, kme, w);
                            const int qi = w * kLsPQ + k % kLsPQ;
                            ls_mbar_wait_backoff(pfull + qi, (uint32_t)(k / kLsPQ) & 1u, p.err, 64);
                            if (lane < 16) v += red[qi * 16 + lane];
                            __syncwarp();
                            if (lane == 0) mbar_arrive(pfree + qi);
                        }
                        const float inv = reinterpret_cast<const volatile float*>(ictl)[5];
                        ls_finish_tile<WT, D>(p, kind, m, ep, tp, tile, v, inv, norm, pos, sl, lane);
                    }
                }
                wbase += wcnt;
            }
            ls_sync_all();  // every tile of the phase finished: the consumers may arrive
        }
        ls_settle(p.err);
        return;
    }

    // =====================================================================
    // consumer warps
    // =====================================================================
    const int ct = threadIdx.x;           // 0 .. kLsWarps * 32 - 1
    const int gq = p.gq;

    // ---- this warp's weight stream: its contiguous share of the CTA's tile-blocks in every
    //      projection phase, cut at row-tile ends and into stages of at most SB blocks; lane 0
    //      keeps kLsWRing stages in flight, across phase boundaries (weights never depend on
    //      the step's activations)
    uint8_t* myring = wring + (size_t)warp * kLsWRing * WS;
    uint64_t* mybar = wfull + warp * kLsWRing;
    int w_ph = 0, w_cur = 0, w_hi = 0, w_k0 = 0, w_nb = 1;
    const uint8_t *w_q = nullptr, *w_s = nullptr;
    auto wnext = [&](const uint8_t*& sq, const uint8_t*& ss, int& n) -> bool {
        for (;;) {
            if (w_cur < w_hi) {
                n = min(min(SB, w_nb - w_k0), w_hi - w_cur);
                sq = w_q + (size_t)w_cur * QB;
                ss = w_s + (size_t)w_cur * kTileSBytes;
                w_cur += n;
                w_k0 += n;
                if (w_k0 == w_nb) w_k0 = 0;
                return true;
            }
            if (++w_ph >= nph) return false;
            const int kind = ls_kind(w_ph, L);
            if (kind == LS_EMB || kind == LS_ATT) continue;
            const LsMat m = ls_mat(p, kind, kind == LS_LM ? L - 1 : (w_ph - 1) / 5);
            int lo, hi;
            ls_range(m, c, G, lo, hi);
            w_cur = lo + (hi - lo) * warp / kLsWarps;
            w_hi = lo + (hi - lo) * (warp + 1) / kLsWarps;
            w_nb = m.nb;
            w_k0 = m.nb > 0 ? w_cur % m.nb : 0;
            w_q = m.q;
            w_s = m.s;
        }
    };
    int wissue = 0;  // stages issued by this warp
    auto wissue_one = [&]() {
        const uint8_t *sq, *ss;
        int n;
        if (!wnext(sq, ss, n)) return;
        if (lane == 0) {
            const int slot = wissue % kLsWRing;
            uint8_t* dst = myring + (size_t)slot * WS;
            mbar_expect_tx(mybar + slot, (uint32_t)(n * (QB + kTileSBytes)));
            bulk_g2s(dst, sq, (uint32_t)(n * QB), mybar + slot);
            bulk_g2s(dst + SB * QB, ss, (uint32_t)(n * kTileSBytes), mybar + slot);
        }
        ++wissue;
    };
    for (int i = 0; i < kLsWRing; ++i) wissue_one();

    pdl_wait();
    pdl_launch_dependents();
    if (ct == 0) {
        const unsigned long long ep = *reinterpret_cast<volatile unsigned long long*>(p.epoch) + 1ull;
        reinterpret_cast<unsigned long long*>(ictl)[0] = ep;
        ictl[2] = p.slots[0];
        ictl[3] = p.pos[ictl[2]];
        ictl[4] = (int)p.tokens[0];
    }
    ls_cbar();
    const unsigned long long target = reinterpret_cast<const unsigned long long*>(ictl)[0] * (unsigned long long)G;
    const int sl = ictl[2], pos = ictl[3];
    const unsigned tok = (unsigned)ictl[4];
    int slot = 0;
    uint32_t round = 0, xphase = 0;
    bool aborted = false;
    int npiece = 0;   // tile pieces this warp queued for the epilogue warps
    int wcons = 0;    // weight stages this warp consumed

    // Wait until every CTA arrived at phase `ph`'s counter.
    auto wait_phase = [&](int ph) {
        if (ct == 0) {
            const long long t0 = clock64();
            while (ld_acquire_u64(p.done + ph) < target) {
                if (ld_volatile_i32(p.err) != 0) break;
                if (clock64() - t0 > kLsSpin) { atomicExch(p.err, kErrDepCounter); break; }
                __nanosleep(20);
            }
        }
        ls_cbar();
    };
    // trace: per-warp ns spent in [0] stage waits, [1] tile-end queue waits, [2] waits for the
    // epilogue warps to finish the phase, [3] phase waits (dependency + records), [4] the whole
    // phase loop
    unsigned* tt_acc = reinterpret_cast<unsigned*>(ictl + 16) + warp * 5;  // (lane 0 adds)
    if (lane == 0)
        for (int k = 0; k < 5; ++k) tt_acc[k] = 0u;
    auto arrive = [&](int ph) {
        const unsigned long long te0 = p.trace ? ls_now() : 0;
        if (p.trace && ct == 0 && ls_kind(ph, L) != LS_ATT) p.trace[((size_t)c * nph + ph) * kLsStamps + 2] = te0;
        ls_sync_all();  // every consumer's and epilogue warp's writes of the phase precede the arrival
        if (p.trace && lane == 0) tt_acc[2] += (unsigned)(ls_now() - te0);
        if (p.trace && ct == 0 && ls_kind(ph, L) != LS_ATT) p.trace[((size_t)c * nph + ph) * kLsStamps + 3] = ls_now();
        if (p.trace && ct == 0) p.trace[((size_t)c * nph + ph) * kLsStamps + 4] = ls_now();
        if (ct == 0) {
            __threadfence();
            if (ph < nph - 1) {
                atomicAdd(p.done + ph, 1ull);  // (result unused: a reduction, no round trip to wait for)
            } else if (atomicAdd(p.done + ph, 1ull) + 1 == target) {  // the step's last arrival
                __threadfence();
                *reinterpret_cast<volatile unsigned long long*>(p.epoch) = target / (unsigned long long)G;
            }
        }
    };
    // the attention ring (K / V chunks from the producer warp)
    // the phase's input records (nb blocks) into `act`; 1/rms from ss_x when `norm`
    auto load_records = [&](const uint8_t* src, int nb, bool norm, int nss) {
        if (ct == 0) {
            mbar_expect_tx(xbar, (uint32_t)ls_rec_bytes(nb));
            bulk_g2s(act, src, (uint32_t)ls_rec_bytes(nb), xbar);
        }
        if (norm && warp == 0) {
            float a = 0.f;
#pragma unroll 8
            for (int i = lane; i < nss; i += 32) a += __ldcg(p.ss_x + i);
            a = warp_sum(a);
            if (lane == 0) reinterpret_cast<float*>(ictl)[5] = 1.f / sqrtf(a / float(p.h) + p.eps);
        }
        if (!ls_mbar_wait_backoff(xbar, xphase, p.err, 64)) aborted = true;
        xphase ^= 1u;
        ls_cbar();
    };

    const uint32_t act_a = smem_u32(act);
    if (ct < 8) ictl[8 + ct] = 0;
    ls_cbar();

    unsigned long long* trace = p.trace ? p.trace + (size_t)c * nph * kLsStamps : nullptr;
    const unsigned long long tl0 = p.trace ? ls_now() : 0;
    for (int ph = 0; ph < nph; ++ph) {
        const int kind = ls_kind(ph, L);
        const int layer = kind == LS_EMB ? 0 : kind == LS_LM ? L - 1 : (ph - 1) / 5;
        if (trace && ct == 0) trace[ph * kLsStamps] = ls_now();
        const unsigned long long tp0 = p.trace ? ls_now() : 0;
        if (ph > 0) wait_phase(ph - 1);
        if (p.trace && lane == 0) tt_acc[3] += (unsigned)(ls_now() - tp0);
        if (kind == LS_EMB || kind == LS_ATT) ls_sync_all();  // (the epilogue warps have nothing to do)
        if (trace && ct == 0 && (kind == LS_EMB || kind == LS_ATT)) trace[ph * kLsStamps + 1] = ls_now();

        // ------------------------------------------------------------ EMB
        if (kind == LS_EMB) {
            const int nblk = p.h / 32;
            for (int b = c + G * warp; b < nblk; b += G * kLsWarps) {
                const int e = 32 * b + lane;
                const float v = tile_value(p.emb_type, p.emb_q, p.emb_s, p.emb_nb, (int)tok, e);
                p.x[e] = v;
                float sq = v * v;
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane == 0) p.ss_x[2 * b] = sq;
                if (lane == 16) p.ss_x[2 * b + 1] = sq;
                dp_lane_record<WT>(v * p.layers[0].attn_norm[e], 0.f, lane & 7, e >> 3, p.rec_x, 1, 2, 4);
            }
            if (c == 0 && ct == 0) atomicAdd(p.counts + (size_t)sl * p.vocab + tok, 1u);
            arrive(ph);
            continue;
        }

        // ------------------------------------------------------------ ATT
        // Chunks [ilo, ihi) of the step's (kv head, CP-position chunk) list. Every consumer
        // warp keeps its own online-softmax state (running max, sum and output of the
        // group's query heads over the positions it owns: pl = warp + 16 i of each chunk),
        // so a chunk needs no CTA barrier; at the end of a run over one kv head the warps'
        // states are merged in shared memory into the CTA's partial, and the last CTA of
        // the head (ticket) merges the partials of its runs and writes the attention output
        // and its records.
        if (kind == LS_ATT) {
            const LsLayer& ly = p.layers[layer];
            const int nch = (pos + 1 + CP - 1) / CP;
            const unsigned I = (unsigned)p.kv_heads * nch;
            const int ilo = ls_lo(I, c, G), ihi = ls_lo(I, c + 1, G);
            if (ilo >= ihi && trace && ct == 0) trace[ph * kLsStamps + 2] = trace[ph * kLsStamps + 3] = ls_now();
            const __half* kg = reinterpret_cast<const __half*>(ly.kc) + (size_t)sl * p.kv_slot_stride;
            const __half* vg = reinterpret_cast<const __half*>(ly.vc) + (size_t)sl * p.kv_slot_stride;
            float* comb = reinterpret_cast<float*>(act);   // [kLsWarps][GM][D + 2] warp states of a run
            float* cw = comb + kLsWarps * GM * (D + 2);    // [kLsWarps][GM] their merge weights
            float o[GM][E], hmx[GM], hsum[GM];
            int run_start = 0;
            int j = ilo / nch, ch = ilo % nch;
            for (int it = ilo; it < ihi; ++it, (++ch == nch ? (ch = 0, ++j) : 0)) {
                if (it == ilo || ch == 0) {
                    // a new kv head: the group's query rows into shared memory, fresh state
                    if (it != ilo) ls_cbar();  // (every warp is done with the previous head's rows)
                    for (int i = ct; i < GM * D; i += kLsWarps * 32)
                        qs[i] = i < gq * D ? __ldcg(p.q + (size_t)j * gq * D + i) : 0.f;
#pragma unroll
                    for (int hh = 0; hh < GM; ++hh) {
#pragma unroll
                        for (int e = 0; e < E; ++e) o[hh][e] = 0.f;
                        hmx[hh] = -INFINITY;
                        hsum[hh] = 0.f;
                    }
                    run_start = ch;
                    ls_cbar();
                }
                const int r0 = ch * CP, nvalid = min(CP, pos + 1 - r0);
                // the chunk ends with this step's row when it holds position pos: the ring stages
                // hold the rows before it (written by earlier steps), and the warp owning that
                // position copies this step's K and V rows (from L2) into the stages' next row
                const bool has_new = r0 + nvalid - 1 == pos;
                // the chunk's K and V stages (consecutive in the ring)
                const int slot_v = slot + 1 == NST ? 0 : slot + 1;
                const uint32_t round_v = slot + 1 == NST ? round + 1 : round;
                {
                    const unsigned long long tw0 = p.trace ? ls_now() : 0;
                    if (!ls_mbar_wait_backoff(full + slot, round & 1u, p.err, 64)) aborted = true;
                    if (!ls_mbar_wait_backoff(full + slot_v, round_v & 1u, p.err, 64)) aborted = true;
                    __syncwarp();
                    if (p.trace && lane == 0) tt_acc[0] += (unsigned)(ls_now() - tw0);
                }
                __half* ks = reinterpret_cast<__half*>(ring + (size_t)slot * kLsStage);
                __half* vs = reinterpret_cast<__half*>(ring + (size_t)slot_v * kLsStage);
                const bool own_new = has_new && (nvalid - 1) % kLsWarps == warp;
                if (own_new) {
                    using R = typename std::conditional<E == 4, uint2, uint32_t>::type;  // E halves
                    const size_t off = ((size_t)j * p.kv_cap + pos) * D + lane * E;
                    const R kk = __ldcg(reinterpret_cast<const R*>(kg + off));
                    const R vv = __ldcg(reinterpret_cast<const R*>(vg + off));
                    *reinterpret_cast<R*>(ks + (size_t)(nvalid - 1) * D + lane * E) = kk;
                    *reinterpret_cast<R*>(vs + (size_t)(nvalid - 1) * D + lane * E) = vv;
                    __syncwarp();
                }
                // this warp's positions, one at a time: score, then the online softmax update
#pragma unroll
                for (int i = 0; i < PPW; ++i) {
                    const int pl = warp + i * kLsWarps;
                    if (pl >= nvalid) break;
                    float kf[E], vf[E];
#pragma unroll
                    for (int e = 0; e < E; e += 2) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(ks + (size_t)pl * D + lane * E + e));
                        const float2 g2 = __half22float2(*reinterpret_cast<const __half2*>(vs + (size_t)pl * D + lane * E + e));
                        kf[e] = f.x; kf[e + 1] = f.y; vf[e] = g2.x; vf[e + 1] = g2.y;
                    }
                    float sc[GM];
#pragma unroll
                    for (int hh = 0; hh < GM; ++hh) {
                        float a = 0.f;
#pragma unroll
                        for (int e = 0; e < E; ++e) a = fmaf(qs[hh * D + lane * E + e], kf[e], a);
                        sc[hh] = a;
                    }
#pragma unroll
                    for (int sh = 16; sh > 0; sh >>= 1)
#pragma unroll
                        for (int hh = 0; hh < GM; ++hh) sc[hh] += __shfl_xor_sync(0xffffffffu, sc[hh], sh);
#pragma unroll
                    for (int hh = 0; hh < GM; ++hh) {
                        const float sv = sc[hh] / p.sqrt_d;
                        const float mn = fmaxf(hmx[hh], sv);
                        const float cs = hmx[hh] == -INFINITY ? 0.f : expf(hmx[hh] - mn);
                        const float pw = expf(sv - mn);
                        hsum[hh] = fmaf(hsum[hh], cs, pw);
#pragma unroll
                        for (int e = 0; e < E; ++e) o[hh][e] = fmaf(o[hh][e], cs, pw * vf[e]);
                        hmx[hh] = mn;
                    }
                }
                // release both stages (the owner's generic writes precede the next bulk copy into them)
                __syncwarp();
                if (lane == 0) {
                    if (own_new) fence_proxy_async_smem();
                    mbar_arrive(empty + slot);
                    mbar_arrive(empty + slot_v);
                }
                slot += 2;
                if (slot >= NST) { slot -= NST; ++round; }

                if (it == ihi - 1 || ch == nch - 1) {
                    // end of this CTA's run over head j: the warps' states into shared memory
#pragma unroll
                    for (int hh = 0; hh < GM; ++hh) {
                        float* st = comb + (warp * GM + hh) * (D + 2);
#pragma unroll
                        for (int e = 0; e < E; ++e) st[lane * E + e] = o[hh][e];
                        if (lane == 0) { st[D] = hmx[hh]; st[D + 1] = hsum[hh]; }
                    }
                    ls_cbar();
                    float* pp = p.apart + ((size_t)j * p.att_maxch + run_start) * (GM * (D + 2));
                    if (warp < gq && lane < kLsWarps) {  // warp hh: the warps' merge weights
                        const int hh = warp;
                        const float m = comb[(lane * GM + hh) * (D + 2) + D];
                        float M = m;
#pragma unroll
                        for (int sh = kLsWarps / 2; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0x0000ffffu, M, sh));
                        const float e = m == -INFINITY ? 0.f : expf(m - M);
                        float S = e * comb[(lane * GM + hh) * (D + 2) + D + 1];
#pragma unroll
                        for (int sh = kLsWarps / 2; sh > 0; sh >>= 1) S += __shfl_xor_sync(0x0000ffffu, S, sh);
                        cw[lane * GM + hh] = e;
                        if (lane == 0) { pp[GM * D + hh] = M; pp[GM * D + GM + hh] = S; }
                    }
                    ls_cbar();
                    for (int i = ct; i < gq * D; i += kLsWarps * 32) {
                        const int hh = i / D;
                        float a = 0.f;
#pragma unroll
                        for (int w = 0; w < kLsWarps; ++w) a = fmaf(cw[w * GM + hh], comb[(w * GM + hh) * (D + 2) + (i % D)], a);
                        pp[i] = a;
                    }
                    ls_cbar();
                    const int jlo = j * nch, jhi = jlo + nch - 1;
                    const int cf = ls_owner(I, jlo, G), cl = ls_owner(I, jhi, G);
                    if (ct == 0) {
                        if (trace) trace[ph * kLsStamps + 2] = ls_now();
                        const unsigned old = atom_add_acq_rel(p.head_tick + j, 1u);
                        ictl[1] = old == (unsigned)(cl - cf);
                    }
                    ls_cbar();
                    if (ictl[1]) {  // the last run of head j: merge every run (CTA order)
                        int nruns = cl - cf + 1;
                        if (nruns > p.att_runs) {  // (the host sizes att_runs for every position; never taken)
                            if (ct == 0) atomicExch(p.err, kErrDepCounter);
                            nruns = p.att_runs;
                        }
                        // the runs' partials in the scratch (run r: CTA cf + r's first chunk of head j)
                        for (int r = ct; r < nruns; r += kLsWarps * 32)
                            roff[r] = (j * p.att_maxch + max(jlo, ls_lo(I, cf + r, G)) - jlo) * (GM * (D + 2));
                        ls_cbar();
                        // per-run weights exp(m_r - M) / S of each head (warp hh, lanes over runs)
                        if (warp < gq) {
                            const int hh = warp;
                            float M = -INFINITY;
                            for (int r = lane; r < nruns; r += 32) M = fmaxf(M, __ldcg(p.apart + roff[r] + GM * D + hh));
                            M = warp_max(M);
                            float S = 0.f;
                            for (int r = lane; r < nruns; r += 32) {
                                const float* q2 = p.apart + roff[r];
                                const float e = expf(__ldcg(q2 + GM * D + hh) - M);
                                wrun[r * GM + hh] = e;
                                S += __ldcg(q2 + GM * D + GM + hh) * e;
                            }
                            S = warp_sum(S);
                            const float is = 1.f / S;
                            for (int r = lane; r < nruns; r += 32) wrun[r * GM + hh] *= is;
                        }
                        ls_cbar();
                        // merged output: the runs' partial outputs, loaded 16 at a time
                        float* obuf = qs;  // [GM][D]
                        for (int i = ct; i < gq * D; i += kLsWarps * 32) {
                            const int hh = i / D;
                            float a = 0.f;
                            for (int r0 = 0; r0 < nruns; r0 += 16) {
                                float ov[16];
#pragma unroll
                                for (int k = 0; k < 16; ++k)
                                    ov[k] = r0 + k < nruns ? __ldcg(p.apart + roff[r0 + k] + i) : 0.f;
#pragma unroll
                                for (int k = 0; k < 16; ++k)
                                    if (r0 + k < nruns) a = fmaf(wrun[(r0 + k) * GM + hh], ov[k], a);
                            }
                            obuf[i] = a;
                        }
                        ls_cbar();
                        // attention output of heads j*gq .. j*gq+gq-1 and its records for O
                        for (int b = warp; b < gq * D / 32; b += kLsWarps) {
                            const float v = obuf[b * 32 + lane];
                            const size_t e = (size_t)j * gq * D + b * 32 + lane;
                            p.attn[e] = v;
                            dp_lane_record<WT>(v, 0.f, lane & 7, (int)(e >> 3), p.rec_attn, 1, 2, 4);
                        }
                        if (ct == 0) p.head_tick[j] = 0u;
                        ls_cbar();
                    }
                    if (trace && ct == 0) trace[ph * kLsStamps + 3] = ls_now();
                }
            }
            arrive(ph);
            continue;
        }

        // ------------------------------------------------------------ projections
        const LsMat m = ls_mat(p, kind, layer);
        const bool norm = kind == LS_QKV || kind == LS_GU || kind == LS_LM;
        if (m.rows > 0) {
            const uint8_t* rsrc = kind == LS_O ? p.rec_attn : kind == LS_DN ? p.rec_act : p.rec_x;
            const unsigned long long tr0 = p.trace ? ls_now() : 0;
            load_records(rsrc, m.nb, norm, p.h / 16);
            if (p.trace && lane == 0) tt_acc[3] += (unsigned)(ls_now() - tr0);
        }
        ls_sync_all();  // the epilogue warps read 1/rms after this
        if (trace && ct == 0) trace[ph * kLsStamps + 1] = ls_now();
        int lo, hi;
        ls_range(m, c, G, lo, hi);
        const int whi = lo + (hi - lo) * (warp + 1) / kLsWarps;
        int cur = lo + (hi - lo) * warp / kLsWarps;
        const int hb = lane >> 4, hu = (lane >> 2) & 3, ht = lane & 3;  // block half, row quad, column group
        if (cur < whi) {  // one piece per row tile this warp's share touches
            for (int tile = cur / m.nb, tlast = (whi - 1) / m.nb; tile <= tlast; ++tile) {
                const int t_end = min(hi, (tile + 1) * m.nb);
                float dacc[4] = {0.f, 0.f, 0.f, 0.f};  // rows 2u, 2u+8, 2u+1, 2u+9 (u = hu)
                while (cur < whi && cur < t_end) {  // this warp's stages inside the tile
                    const int k0 = cur - tile * m.nb;
                    const int n = min(min(SB, m.nb - k0), whi - cur);
                    const int wslot = wcons % kLsWRing;
                    const unsigned long long tw0 = p.trace ? ls_now() : 0;
                    if (!ls_mbar_wait_backoff(mybar + wslot, (uint32_t)(wcons / kLsWRing) & 1u, p.err, 64)) aborted = true;
                    if (p.trace && lane == 0) tt_acc[0] += (unsigned)(ls_now() - tw0);
                    const uint32_t sq = smem_u32(myring + (size_t)wslot * WS);
                    const uint32_t ssc = sq + SB * QB;
                    const uint32_t xr = act_a + (uint32_t)k0 * kLsRec;
                    // the two half warps take alternate blocks of the stage
                    if (n == SB) {
#pragma unroll
                        for (int jb = 0; jb < SB; jb += 2) {
                            const int j = jb + hb;
                            ls_block_dp4<WT>(sq + j * QB, ssc + j * kTileSBytes, xr + j * kLsRec, hu, ht, dacc);
                        }
                    } else {
                        for (int jb = 0; jb < n; jb += 2) {
                            const int j = jb + hb;
                            if (j < n)
                                ls_block_dp4<WT>(sq + j * QB, ssc + j * kTileSBytes, xr + j * kLsRec, hu, ht, dacc);
                        }
                    }
                    __syncwarp();
                    ++wcons;
                    if (lane == 0) fence_proxy_async_smem();  // the reads of this slot precede its refill
                    wissue_one();
                    cur += n;
                }
                // ---- this warp's piece of the tile into its queue: a row's sums are spread over
                //      its four column-group lanes and the two half warps
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    dacc[r] += __shfl_xor_sync(0xffffffffu, dacc[r], 1);
                    dacc[r] += __shfl_xor_sync(0xffffffffu, dacc[r], 2);
                    dacc[r] += __shfl_xor_sync(0xffffffffu, dacc[r], 16);
                }
                const int qi = warp * kLsPQ + npiece % kLsPQ;
                const uint32_t use = (uint32_t)(npiece / kLsPQ);
                const unsigned long long tq0 = p.trace ? ls_now() : 0;
                if (use > 0 && !ls_mbar_wait_backoff(pfree + qi, (use - 1) & 1u, p.err, 64)) aborted = true;
                if (p.trace && lane == 0) tt_acc[1] += (unsigned)(ls_now() - tq0);
                if (lane < 16 && ht == 0) {
                    float* rp = red + qi * 16 + 2 * hu;
                    rp[0] = dacc[0];
                    rp[8] = dacc[1];
                    rp[1] = dacc[2];
                    rp[9] = dacc[3];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(pfull + qi);
                ++npiece;
            }
        }
        arrive(ph);
    }
    if (p.trace) {
        if (lane == 0) {  // [CTA][warp][5]
            tt_acc[4] = (unsigned)(ls_now() - tl0);
            unsigned long long* st = p.trace + (size_t)G * nph * kLsStamps + ((size_t)c * kLsWarps + warp) * 5;
            for (int k = 0; k < 5; ++k) st[k] = tt_acc[k];
        }
    }
    (void)aborted;
    ls_settle(p.err);
}

}  // namespace laic
