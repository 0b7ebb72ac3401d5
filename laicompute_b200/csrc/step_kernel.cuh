// Decode step of one sequence as one persistent kernel (the batch-1 latency path).
//
// Replaces the per-layer launches of LlamaRuntime::step (reference
// src/inference_v2.cpp:31) for one sequence whose projections are all Q4_0 or
// all Q8_0, with an FP16 KV cache. One CTA per SM (a cooperative launch, so all
// CTAs are resident) runs, for every layer,
//   QKV   rmsnorm + fused [Wq;Wk;Wv] + RoPE + K/V append      (integer variant)
//   ATTN  tensor-core attention over 128-position chunks     (four warps)
//   O     Wo attn, added into the residual
//   GU    rmsnorm + interleaved [Wgate;Wup] + SwiGLU
//   DOWN  Wdown act, added into the residual
// with a grid barrier after each phase (its outputs are the next one's inputs).
//
// The weights never depend on the previous phase, so each warp streams ONE
// continuous sequence of tile-block stages through its shared-memory ring for
// the whole step: the stages of phase m+1 are already in flight while phase m
// finishes, the barrier resolves and the next activation records are built.
// Within a projection phase the work split is the team kernel's (whole 16-row
// tiles per CTA, teams of warps over K); the lm_head and the sampler stay
// separate kernels.
//
// Every wait is bounded (~1 s of clock): on timeout the kernel records the
// failure in `err` and carries on to the end, so it always terminates.
#pragma once
#include "attention.cuh"
#include "mv_streamk.cuh"

namespace laic {

struct StepMat {
    const uint8_t* q;
    const uint8_t* s;
};
struct StepLayer {
    StepMat qkv, o, gu, down;
    const float* attn_norm;
    const float* ffn_norm;
    void* kc;  // this layer's K cache
    void* vc;  // this layer's V cache
};
struct StepParams {
    const StepLayer* layers;
    int L;
    int h, F, hq, kv, D, heads, kv_heads, rope_pairs;
    float eps, sqrt_d;
    float *x, *q, *attn, *act;
    const float2* rope_cs;
    const int* slots;  // [1]
    const int* pos;    // [max_seqs]
    long long kv_slot_stride;
    int kv_cap;
    float* part;        // attention chunk partials
    unsigned* counters; // [kv_heads] tickets, zero between launches
    unsigned* bar;      // grid barrier arrivals, zero at launch
    int* err;
    // activation digit records made by the producing phase's epilogue (see dp_lane_record)
    uint8_t* rec_x;     // [h / 8][32 B]: residual x times the next rmsnorm weight (next GU or QKV)
    uint8_t* rec_act;   // [F / 8][32 B]: SwiGLU output (next DOWN)
    float* ss_x;        // [h / 8] sums of squares of x per 8-column group (the next rmsnorm)
};

enum : int { SK_QKV = 0, SK_O = 1, SK_GU = 2, SK_DOWN = 3 };

// Shape of projection `kind` (every layer has the same).
struct StepMv {
    int rows, in, nb, ntiles;
};
__device__ __forceinline__ StepMv step_mv(const StepParams& p, int kind) {
    StepMv m;
    m.rows = kind == SK_QKV ? p.hq + 2 * p.kv : kind == SK_GU ? 2 * p.F : p.h;
    m.in = kind == SK_O ? p.hq : kind == SK_DOWN ? p.F : p.h;
    m.nb = m.in / 32;
    m.ntiles = (m.rows + 15) / 16;
    return m;
}
__device__ __forceinline__ StepMat step_mat(const StepLayer& ly, int kind) {
    return kind == SK_QKV ? ly.qkv : kind == SK_O ? ly.o : kind == SK_GU ? ly.gu : ly.down;
}

// All CTAs arrive, then leave together; writes before arrival are visible after.
__device__ __forceinline__ void step_grid_sync(unsigned* bar, unsigned target, int* err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned old = atomicAdd(bar, 1u);
        if (old + 1 < target) {  // not the last to arrive: wait for the rest
            const long long t0 = clock64();
            unsigned v;
            while (true) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
                if (v >= target) break;
                if (clock64() - t0 > 2000000000LL) { atomicExch(err, kErrGridBarrier); break; }
            }
        }
    }
    __syncthreads();
}

// Shared memory of the step kernel: rings, a region shared by the activation
// records and the attention chunk buffers, partial slots, tickets, barriers.
__host__ __device__ inline size_t step_union_bytes(int type, int nb_max, int D) {
    const size_t xs = (size_t)nb_max * kDpRecBytes;
    const size_t at = attn_chunk_smem(D);
    return xs > at ? xs : at;
}
__host__ __device__ inline size_t step_smem_bytes(int type, int nb_max, int D) {
    const size_t rings = (size_t)kSkWarps * sk_stages(type) * sk_stage_bytes(type);
    const size_t parts = (size_t)kSkWarps * kSkSlots * 16 * 4;
    return rings + step_union_bytes(type, nb_max, D) + parts + sk_small_bytes(1) +
           (size_t)kSkWarps * sk_stages(type) * 8 + 8;  // + the activation-copy barrier
}

template <int WT, int D, int GMAX>
__global__ void __launch_bounds__(kSkWarps * 32, 1) step_kernel(const StepParams p) {
    constexpr int QB = tile_qbytes(WT);
    constexpr int SB = kTileSBytes;
    constexpr int KB = sk_kb(WT);
    constexpr int R = sk_stages(WT);
    constexpr int STAGE = sk_stage_bytes(WT);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int nb_max = max(max(p.h, p.hq), p.F) / 32;

    uint8_t* ring = smem + warp * R * STAGE;
    uint8_t* uni = smem + kSkWarps * R * STAGE;  // activation records | attention chunk
    float* parts = reinterpret_cast<float*>(uni + step_union_bytes(WT, nb_max, D));  // [warp][slot][16]
    uint8_t* small = reinterpret_cast<uint8_t*>(parts + kSkWarps * kSkSlots * 16);
    int* tickets = reinterpret_cast<int*>(small);
    int* merged = tickets + kSkWarps * kSkSlots;
    float* wstat = reinterpret_cast<float*>(merged + kSkWarps * kSkSlots);
    float* inv = wstat + kSkWarps * 2;
    uint64_t* bars = reinterpret_cast<uint64_t*>(small + sk_small_bytes(1)) + warp * R;
    uint64_t* xbar = reinterpret_cast<uint64_t*>(small + sk_small_bytes(1)) + kSkWarps * R;  // activation copies
    uint32_t xpar = 0;
    const int grid = gridDim.x, bid = blockIdx.x;
    const int nmv = 4 * p.L;  // projection phases in stream order: layer-major, kind-minor

    // ---- this warp's stage stream over all projection phases
    struct Cur {
        int m, ti, st;        // phase, tile index among this warp's tiles, stage within the slice
        int t0, teams, ntl;   // first tile, tile step, tiles of this warp in the phase
        int b_lo, b_hi, spt;  // K slice (blocks) and stages per tile
        const uint8_t *q, *s;
        int nb;
    };
    auto setup = [&](Cur& u, int m) {
        // move to phase m or the first later phase where this warp has work
        for (; m < nmv; ++m) {
            const int kind = m & 3;
            const StepMv mv = step_mv(p, kind);
            const int k = sk_team(mv.nb), teams = kSkWarps / k, team = warp / k, wi = warp % k;
            const int t_lo = (int)((long long)bid * mv.ntiles / grid), t_hi = (int)((long long)(bid + 1) * mv.ntiles / grid);
            int ntl = 0;
            for (int t = t_lo + team; t < t_hi; t += teams) ++ntl;
            const int b_lo = wi * mv.nb / k, b_hi = (wi + 1) * mv.nb / k;
            const int spt = (b_hi - b_lo + KB - 1) / KB;
            if (ntl > 0 && spt > 0) {
                const StepMat mat = step_mat(p.layers[m >> 2], kind);
                u = Cur{m, 0, 0, t_lo + team, teams, ntl, b_lo, b_hi, spt, mat.q, mat.s, mv.nb};
                return;
            }
        }
        u.m = nmv;
    };
    Cur iss;  // next stage to issue (lane 0)
    int iss_slot = 0;
    setup(iss, 0);
    auto issue = [&]() -> bool {
        if (iss.m >= nmv) return false;
        const int t = iss.t0 + iss.ti * iss.teams;
        const int b0 = iss.b_lo + iss.st * KB;
        const int n = min(KB, iss.b_hi - b0);
        const size_t first = (size_t)t * iss.nb + b0;
        uint8_t* dst = ring + iss_slot * STAGE;
        mbar_expect_tx(bars + iss_slot, (uint32_t)(n * (QB + SB)));
        bulk_g2s(dst, iss.q + first * QB, (uint32_t)(n * QB), bars + iss_slot);
        bulk_g2s(dst + KB * QB, iss.s + first * SB, (uint32_t)(n * SB), bars + iss_slot);
        if (++iss_slot == R) iss_slot = 0;
        if (++iss.st == iss.spt) {
            iss.st = 0;
            if (++iss.ti == iss.ntl) setup(iss, iss.m + 1);
        }
        return true;
    };
    int issued = 0, consumed = 0;
    if (lane == 0) {
        for (int r = 0; r < R; ++r) mbar_init(bars + r, 1);
        if (warp == 0) mbar_init(xbar, 1);
        mbar_fence_init();
        for (int r = 0; r < R && issue(); ++r) ++issued;
    }
    __syncwarp();

    int slot = 0;
    uint32_t phase = 0;
    bool aborted = false;
    unsigned nbar = 0;  // grid barriers passed
    const int xwarp_rec = c * 32;  // this lane's 8-column group inside a block record

    for (int l = 0; l < p.L; ++l) {
        const StepLayer& ly = p.layers[l];
        for (int kind = 0; kind < 5; ++kind) {
            if (kind == 1) {
                // ---------------- attention: (kv head, chunk) items over the CTAs, four warps each
                const int slot_s = p.slots[0];
                const int n = p.pos[slot_s] + 1;
                const int nch = (n + kAttnChunk - 1) / kAttnChunk;
                if (threadIdx.x < kAttnWarps * 32) {
                    AttnParams ap{};
                    ap.q = p.q; ap.ldq = p.hq; ap.out = p.attn; ap.ldo = p.hq;
                    ap.kc = ly.kc; ap.vc = ly.vc; ap.slot_stride = p.kv_slot_stride; ap.cap = p.kv_cap;
                    ap.heads = p.heads; ap.kv_heads = p.kv_heads; ap.slots = p.slots; ap.pos = p.pos;
                    ap.nsplit = nch; ap.part = p.part; ap.counters = p.counters; ap.sqrt_d = p.sqrt_d; ap.err = p.err;
                    for (int it = bid; it < p.kv_heads * nch; it += grid)
                        attn_mma_body<D, GMAX, false>(ap, it / p.kv_heads, it % p.kv_heads, 0, uni, threadIdx.x, 2);
                }
                step_grid_sync(p.bar, ++nbar * (unsigned)grid, p.err);
                continue;
            }
            const int mk = kind == 0 ? SK_QKV : kind - 1;  // O, GU, DOWN
            const StepMv mv = step_mv(p, mk);
            for (int i = threadIdx.x; i < 2 * kSkWarps * kSkSlots; i += blockDim.x) tickets[i] = 0;  // and merged[]
            // the input records: built here for layer 0's QKV (x from the embedding) and for O (the
            // attention output); copied whole from the producing epilogue's records otherwise, with
            // the rmsnorm's 1/rms (a scalar) applied to the outputs
            float oscale = 1.f;
            if ((mk == SK_QKV && l == 0) || mk == SK_O) {
                dp_build_records<WT>(mk == SK_O ? p.attn : p.x, mk == SK_O ? nullptr : ly.attn_norm, p.eps, mv.in, uni,
                                     wstat, inv);  // ends with a CTA barrier
            } else {
                if (threadIdx.x == 0) {
                    fence_proxy_async_smem();  // earlier generic accesses of the region precede the copy
                    const uint32_t bytes = (uint32_t)mv.nb * kDpRecBytes;
                    mbar_expect_tx(xbar, bytes);
                    bulk_g2s(uni, mk == SK_DOWN ? p.rec_act : p.rec_x, bytes, xbar);
                }
                if (mk != SK_DOWN) {  // 1/rms from the per-group sums of squares, in a fixed order
                    float a = 0.f;
                    for (int gi = threadIdx.x; gi < p.h / 8; gi += blockDim.x) a += __ldcg(p.ss_x + gi);
                    a = warp_sum(a);
                    if (lane == 0) wstat[warp * 2] = a;
                    __syncthreads();
                    float tot = 0.f;
                    for (int w = 0; w < kSkWarps; ++w) tot += wstat[w * 2];
                    oscale = 1.f / sqrtf(tot / float(p.h) + p.eps);
                }
                if (!mbar_wait(xbar, xpar, p.err)) aborted = true;
                xpar ^= 1u;
                __syncthreads();
            }

            // this warp's tiles and K slice in this phase (the issue cursor walked the same)
            const int k = sk_team(mv.nb), teams = kSkWarps / k, team = warp / k, wi = warp % k, leader = team * k;
            const int t_lo = (int)((long long)bid * mv.ntiles / grid), t_hi = (int)((long long)(bid + 1) * mv.ntiles / grid);
            const int b_lo = wi * mv.nb / k, b_hi = (wi + 1) * mv.nb / k;
            const int spt = (b_hi - b_lo + KB - 1) / KB;
            const uint32_t xr0 = smem_u32(uni) + xwarp_rec;
            int ti = 0;
            for (int t = t_lo + team; t < t_hi && spt > 0; t += teams, ++ti) {
                float acc[2] = {0.f, 0.f};
                for (int st = 0; st < spt; ++st) {
                    if (!aborted && !mbar_wait(bars + slot, phase, p.err)) aborted = true;
                    const int b0 = b_lo + st * KB;
                    const int n = aborted ? 0 : min(KB, b_hi - b0);
                    const uint32_t sq = smem_u32(ring) + slot * STAGE;
                    const uint32_t ssc = sq + KB * QB;
                    const uint32_t xr = xr0 + b0 * kDpRecBytes;
                    if (n == KB) {
#pragma unroll
                        for (int j = 0; j < KB; ++j) tile_block_dp<WT>(sq + j * QB, ssc + j * SB, xr + j * kDpRecBytes, lane, acc);
                    } else {
                        for (int j = 0; j < n; ++j) tile_block_dp<WT>(sq + j * QB, ssc + j * SB, xr + j * kDpRecBytes, lane, acc);
                    }
                    __syncwarp();
                    ++consumed;
                    if (lane == 0 && !aborted) {
                        fence_proxy_async_smem();  // this warp's reads of the slot precede its refill
                        if (issue()) ++issued;
                    }
                    if (++slot == R) { slot = 0; phase ^= 1u; }
                }
                // ---- the tile's partial: lanes of a row add their groups; the team's last warp merges
                const int tslot = ti % kSkSlots;
                float* mine = parts + ((size_t)warp * kSkSlots + tslot) * 16;
                if (ti >= kSkSlots) {
                    if (lane == 0) {
                        const long long c0 = clock64();
                        while (*reinterpret_cast<volatile int*>(merged + leader * kSkSlots + tslot) < ti - kSkSlots + 1) {
                            if (clock64() - c0 > 2000000000LL) { atomicExch(p.err, kErrTeamMerge); break; }
                        }
                    }
                    __syncwarp();
                }
                float r0 = acc[0], r1 = acc[1];
                r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
                r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
                r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
                r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
                if (c == 0) { mine[g] = r0; mine[g + 8] = r1; }
                __threadfence_block();
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(tickets + leader * kSkSlots + tslot, 1) == k - 1;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;
                __threadfence_block();
                float v = 0.f;
                if (lane < 16)
                    for (int w = 0; w < k; ++w) v += parts[((size_t)(leader + w) * kSkSlots + tslot) * 16 + lane];
                const float vo = __shfl_xor_sync(0xffffffffu, v, 1);  // the other row of the pair
                if (lane == 0) {
                    tickets[leader * kSkSlots + tslot] = 0;
                    __threadfence_block();
                    merged[leader * kSkSlots + tslot] = ti + 1;
                }
                const int r = t * 16 + lane;
                v *= oscale;
                const float vo2 = vo * oscale;
                if (mk == SK_O || mk == SK_DOWN) {
                    // residual add; then the records of x * (next rmsnorm weight) and its group sums of squares
                    const bool live = lane < 16 && r < mv.rows;
                    const float xn = live ? __ldcg(p.x + r) + v : 0.f;
                    if (live) p.x[r] = xn;
                    const float* nwn = mk == SK_O ? ly.ffn_norm : (l + 1 < p.L ? p.layers[l + 1].attn_norm : nullptr);
                    if (nwn) {
                        const float ssg = dp_lane_record<WT>(live ? xn * nwn[r] : 0.f, xn * xn, lane & 7,
                                                                live ? (r >> 3) : -1, p.rec_x, 1, 2, 4);
                        if (live && (lane & 7) == 0) p.ss_x[r >> 3] = ssg;
                    }
                } else if (mk == SK_GU) {
                    // row 2o = gate o, row 2o+1 = up o: act[o] = silu(gate) * up; the tile's 8 values are one group
                    const bool live = lane < 16 && (lane & 1) == 0 && r < mv.rows;
                    const float av = live ? (v / (1.f + expf(-v))) * vo2 : 0.f;
                    if (live) p.act[r >> 1] = av;
                    dp_lane_record<WT>(av, 0.f, lane >> 1, live ? t : -1, p.rec_act, 2, 4, 8);
                } else if (lane < 16 && r < mv.rows) {  // QKV: RoPE on q and k, then q out and K/V appended
                        const int sl = p.slots[0], ps = p.pos[sl];
                        int rr = r, region = 0;
                        if (rr >= p.hq) { rr -= p.hq; region = 1; if (rr >= p.kv) { rr -= p.kv; region = 2; } }
                        const int d = rr % p.D;
                        float o = v;
                        if (region < 2 && d < 2 * p.rope_pairs) {
                            const float2 cs = p.rope_cs[(size_t)ps * p.rope_pairs + (d >> 1)];
                            // adjacent-pair rotation, unfused to keep the reference's rounding
                            if ((d & 1) == 0) o = __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(vo2, cs.y));
                            else o = __fadd_rn(__fmul_rn(vo2, cs.y), __fmul_rn(v, cs.x));
                        }
                        if (region == 0) {
                            p.q[rr] = o;
                        } else {
                            __half* base = reinterpret_cast<__half*>(region == 1 ? ly.kc : ly.vc);
                            base[(size_t)sl * p.kv_slot_stride + ((size_t)(rr / p.D) * p.kv_cap + ps) * p.D + d] =
                                __float2half_rn(o);
                        }
                }
                __syncwarp();
            }
            step_grid_sync(p.bar, ++nbar * (unsigned)grid, p.err);
        }
    }
    if (aborted && lane == 0) {
        // leave only after the copies still in flight into this warp's ring have landed
        for (int s = max(0, issued - R); s < issued; ++s) mbar_wait(bars + (s % R), (uint32_t)(s / R) & 1u, p.err);
    }
    (void)consumed;
}

}  // namespace laic
