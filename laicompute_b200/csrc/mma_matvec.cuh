// Dequant-fused matrix-vector / skinny-GEMM for decode on sm_100a.
//
// Replaces LlamaRuntime::matvec (reference src/inference_v2.cpp:29) and its two
// row-dot paths, quant_dot (:21, quant_v2::value per element) and dot_cached
// (:22, compute::dot_f16), for 1..64 sequences. Each projection of a layer is
// one launch that also carries the elementwise work around it:
//   prologue  rmsnorm of the residual (src/inference_v2.cpp:24 and :30)
//   epilogue  store | residual add (compute::axpy_f32, src/compute_dot.cpp:64-72)
//             | SwiGLU (gate/up rows interleaved, :23 and :31)
//             | QKV: RoPE (:25) on q and k, then K/V appended to the device cache
//
// Data path.
//  * Weights live in a "fragment tile" layout built once at upload: 16 rows x
//    32 columns (one GGUF block column) form a tile-block whose bytes are laid
//    out so that lane L of a warp reads exactly the A-operand fragment of
//    mma.m16n8k16 it needs (rows g and g+8, g = L/4, for 8 of the 32 columns).
//    Block quants and binary16 scales keep their file values.
//  * A producer warp streams the tile-blocks of the CTA's work into a shared
//    memory ring with 1-D bulk TMA copies (cp.async.bulk + mbarrier), issued
//    before the programmatic-dependent-launch wait: weights never depend on
//    the previous kernel, so the stream starts while that kernel drains.
//  * Consumer warps turn quants into exact binary16 integers with one
//    AND/OR per pair (0x6400 exponent trick) and one packed subtract, and run
//    mma.sync m16n8k16 (fp16 in, fp32 accumulate) against the activations,
//    which are split into binary16 hi + lo parts (hi + lo carries 22 bits of
//    the fp32 value): y = sum_blocks d * (q . x_hi + q . x_lo) in fp32.
//  * The K dimension may be split across CTAs; the last CTA of a row tile
//    (atomic ticket, no spinning) adds the partials in a fixed order and runs
//    the epilogue, so results are deterministic.
#pragma once
#include "common.cuh"
#include "tiles.cuh"

namespace laic {

enum : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

constexpr int kConsumerWarps = 8;
constexpr int kMvThreads = (kConsumerWarps + 1) * 32;


struct MvParams {
    const uint8_t* q;          // [ntiles][nb][tile_qbytes]
    const uint8_t* s;          // [ntiles][nb][32]   (Q4_0/Q8_0)
    int rows, ntiles, in, nb;
    int nseq;
    const float* x;            // input [nseq][ldx]
    int ldx;
    const float* norm_w;       // rmsnorm weight [in] (nullptr: no norm)
    float eps;
    int nk, kr, kb, stages;    // K splits, blocks per split, blocks per ring stage, ring depth
    int sgrp;                  // tile kernel: sequences per CTA group (grid.y = groups)
    float* part;               // split-K partials [ntiles][nk][16][nseq] (scratch)
    unsigned* tile_cnt;        // [ntiles][groups] tickets, zero between launches (scratch)
    int* err;                  // set when a bounded wait runs out
    float* out;                // epilogue output
    int ldo;
    // EPI_QKV
    int q_rows, kv_rows, head_dim, rope_pairs;
    const float2* rope_cs;     // [ctx][rope_pairs] (cos, sin)
    const int* slots;          // [nseq]
    const int* pos;            // [max_seqs]
    void* kc;                  // this layer's K cache
    void* vc;                  // this layer's V cache
    long long kv_slot_stride;  // elements between slots
    int kv_cap;
    // tile kernel: activations already split by xprep_kernel
    const uint8_t* xg;         // records (rec_off): [nb][hi, lo][nseq][4][16 B] binary16 in fragment order
    const float* xinvg;        // [nk][nseq] power-of-two scale of each K split
    // tile kernel, records made by the producing kernel instead of xprep_kernel (then unscaled):
    int scale_mode;            // 0: xinvg; 1: rmsnorm 1/rms from `ss`; 2: unit scale
    const float* ss;           // [ss_tiles][nseq] partial sums of squares of the rmsnorm input
    int ss_tiles, ss_n;        // partials per sequence, elements per row
    // tile kernel EPI_ADD / EPI_SWIGLU: records of the output for the next tile-kernel projection
    uint8_t* rec_out;          // records (rec_off) of rows or rows/2 elements (nullptr: none)
    const float* rec_w;        // EPI_ADD: the next rmsnorm weight (records of out * w), or nullptr
    float* ss_out;             // EPI_ADD: [row tiles][nseq] sums of squares of the new residual
    // team kernel, one sequence (integer variant): scale_mode 1 or 2 with ss, ss_tiles, ss_n as
    // above: it builds the records of x * norm_w itself and scales the rows by the rmsnorm's 1/rms
    // from the partial sums (EPI_ADD writes them to ss_out for the next projection)
    // team kernel: its split, computed on the host (the kernel takes no divisions): warps per
    // team, teams per CTA and ceil(65536 / team_k) (warp / team_k = warp * team_inv >> 16);
    // tiles per CTA (tq, one more in the first tr CTAs) and blocks per warp's slice of a tile
    // (sq, one more for the first sr warps of a team)
    int team_k, team_n, team_inv, tq, tr, sq, sr;
};

// Activation records (the tile and wide kernels' B operands): per GGUF block column bl
// a hi plane, then a lo plane, each [nseq][4 column groups c][8 binary16 in fragment
// order]. Byte offset of (bl, part, s, c), part 0 = hi, 1 = lo. The eight lanes of one
// shared-memory phase (two sequences x four groups) then read 128 consecutive bytes.
__host__ __device__ __forceinline__ size_t rec_off(int bl, int part, int nseq, int s, int c) {
    return (((size_t)bl * 2 + part) * nseq + s) * 64 + (size_t)c * 16;
}

// Record of element e of sequence s (binary16 hi + lo), the layout xprep_kernel writes.
__device__ __forceinline__ void store_act_record(uint8_t* rec, int nseq, int e, int s, float v) {
    const int bl = e >> 5, c = (e >> 3) & 3, k = frag_pos(e & 7);
    const __half hi = __float2half_rn(v);
    reinterpret_cast<__half*>(rec + rec_off(bl, 0, nseq, s, c))[k] = hi;
    reinterpret_cast<__half*>(rec + rec_off(bl, 1, nseq, s, c))[k] = __float2half_rn(v - __half2float(hi));
}

// Activation preparation for the tile kernel (one launch before it).
struct XPrepParams {
    const float* x;            // [nseq][ldx]
    int ldx;
    const float* norm_w;       // rmsnorm weight [in] (nullptr: no norm)
    float eps;
    int in, nb, nseq;
    int kr;                    // blocks per K split of the consuming matvec
    uint8_t* xg;               // out: records (rec_off)
    float* xinv;               // out: [nk][nseq]
};

// ---------------------------------------------------------------------------
// PTX helpers: mbarrier, bulk copy, mma
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait that lets the hardware suspend the thread (up to ~0.1 ms) until the
// phase completes, so waiting warps do not take issue slots from working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}
// Wait for a barrier phase with a time limit (~1 s of SM clocks); on timeout
// record the failure and return false so the caller can leave cleanly.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (clock64() - t0 > 2000000000LL) {
            atomicExch(err, kErrMbarrier);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// A sequence group's slice of nblk blocks of activation records (from block b0) into
// shared memory, 16 bytes per thread and step, by the n threads tid 0..n-1 (cp.async;
// the caller waits and synchronises).
__device__ __forceinline__ void load_rec_slice(uint8_t* xs, const uint8_t* xg, int b0, int nblk, int B, int s0, int Bl,
                                               int tid, int n) {
    const int per_plane = Bl * 4;
    for (int i = tid; i < nblk * 2 * per_plane; i += n) {
        const int c = i & 3, s = (i >> 2) % Bl, plane = i / per_plane;
        cp_async16(xs + rec_off(plane >> 1, plane & 1, Bl, s, c), xg + rec_off(b0 + (plane >> 1), plane & 1, B, s0 + s, c));
    }
    cp_async_commit();
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t a0, const uint32_t a1, const uint32_t a2,
                                         const uint32_t a3, const uint32_t b0, const uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same product with a zero accumulator input (no zeroed registers to set up).
__device__ __forceinline__ void mma16816_z(float (&d)[4], const uint32_t a0, const uint32_t a1, const uint32_t a2,
                                           const uint32_t a3, const uint32_t b0, const uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}
// Accumulating product without the volatile qualifier, so the compiler may interleave independent tiles.
__device__ __forceinline__ void mma16816_acc(float (&d)[4], const uint32_t a0, const uint32_t a1, const uint32_t a2,
                                             const uint32_t a3, const uint32_t b0, const uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b), *reinterpret_cast<__half2*>(&c));
    return *reinterpret_cast<uint32_t*>(&r);
}

// Q4_0 word (8 nibbles, elements e0..e7 of one row's 8-column group) ->
// four half2 registers (e0,e4) (e1,e5) (e2,e6) (e3,e7) holding q-8 exactly.
__device__ __forceinline__ void decode_q4(uint32_t w, uint32_t (&r)[4]) {
    const uint32_t M = 0x64006400u;                 // binary16 1024 in both halves
    const uint32_t k1032 = 0x64086408u;             // 1032
    const uint32_t k1_16 = 0x2C002C00u;             // 1/16
    const uint32_t km72 = 0xD480D480u;              // -72
    const uint32_t w8 = w >> 8;
    r[0] = h2_sub((w & 0x000F000Fu) | M, k1032);            // (1024+n) - 1032
    r[1] = h2_fma((w & 0x00F000F0u) | M, k1_16, km72);      // (1024+16n)/16 - 72
    r[2] = h2_sub((w8 & 0x000F000Fu) | M, k1032);
    r[3] = h2_fma((w8 & 0x00F000F0u) | M, k1_16, km72);
}
// Q8_0: 8 int8 of one row in fragment order (e0 e4 e1 e5 | e2 e6 e3 e7) -> four half2 = q.
__device__ __forceinline__ void decode_q8(uint32_t u0, uint32_t u1, uint32_t (&r)[4]) {
    const uint32_t C = 0x64646464u, k1152 = 0x64806480u;  // 1024 + 128
    u0 ^= 0x80808080u;
    u1 ^= 0x80808080u;
    r[0] = h2_sub(__byte_perm(u0, C, 0x4140), k1152);
    r[1] = h2_sub(__byte_perm(u0, C, 0x4342), k1152);
    r[2] = h2_sub(__byte_perm(u1, C, 0x4140), k1152);
    r[3] = h2_sub(__byte_perm(u1, C, 0x4342), k1152);
}

template <typename KV> __device__ __forceinline__ KV kv_from(float v);
template <> __device__ __forceinline__ __half kv_from<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float kv_from<float>(float v) { return v; }

// Host-side sizing shared with the launcher.
__host__ __device__ constexpr int mv_ring_bytes(int type, int kb, int stages) {
    return stages * kb * (tile_qbytes(type) + (type == T_F16 ? 0 : kTileSBytes));
}

// 1/scale of each sequence of a group into xinv[0 .. Bl): xprep's power-of-two scale of the
// K split (mode 0), the rmsnorm of the whole row from the producers' partial sums of
// squares (mode 1), or 1 (mode 2). Mode 1 spreads a sequence's partial sums over tps
// threads of one warp (a power of two) and adds them in a fixed tree order.
__device__ __forceinline__ void seq_scales(const MvParams& p, int k_split, int s0, int Bl, float* xinv, int tid, int n) {
    if (p.scale_mode != 1) {
        for (int sl = tid; sl < Bl; sl += n)
            xinv[sl] = p.scale_mode == 0 ? p.xinvg[(size_t)k_split * p.nseq + s0 + sl] : 1.f;
        return;
    }
    int tps = 32;
    while (tps > 1 && tps * Bl > n) tps >>= 1;
    const int part = tid % tps;
    for (int sl0 = 0; sl0 < Bl; sl0 += n / tps) {  // the same trip count in every thread
        const int sl = sl0 + tid / tps;
        float a = 0.f;
        if (sl < Bl) {
            const float* src = p.ss + s0 + sl;
            int t = part;
            for (; t + 3 * tps < p.ss_tiles; t += 4 * tps) {
                const float v0 = __ldcg(src + (size_t)t * p.nseq), v1 = __ldcg(src + (size_t)(t + tps) * p.nseq);
                const float v2 = __ldcg(src + (size_t)(t + 2 * tps) * p.nseq);
                const float v3 = __ldcg(src + (size_t)(t + 3 * tps) * p.nseq);
                a += (v0 + v1) + (v2 + v3);
            }
            for (; t < p.ss_tiles; t += tps) a += __ldcg(src + (size_t)t * p.nseq);
        }
        for (int o = tps >> 1; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (sl < Bl && part == 0) xinv[sl] = 1.f / sqrtf(a / float(p.ss_n) + p.eps);
    }
}

// ---------------------------------------------------------------------------
// the kernel: NT n-tiles of 8 sequences (NT*8 >= nseq)
// ---------------------------------------------------------------------------
template <int WT, int NT, int EPI, typename KV>
__global__ void __launch_bounds__(kMvThreads, 1) mv_mma_kernel(const MvParams p) {
    constexpr int QB = tile_qbytes(WT);
    constexpr int SB = WT == T_F16 ? 0 : kTileSBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int B = p.nseq;                   // all sequences (the global layouts)
    const int s0 = blockIdx.y * p.sgrp;     // this CTA's sequence group: s0 .. s0 + Bl - 1
    const int Bl = min(p.sgrp, B - s0);
    const int stage_bytes = p.kb * (QB + SB);

    uint8_t* ring = smem;
    uint8_t* xs = ring + p.stages * stage_bytes;                            // records of [kr] blocks x [Bl]
    float* red = reinterpret_cast<float*>(xs + (size_t)p.kr * p.sgrp * 128);  // [8 warps][16][NT*8]
    float* fin = red + kConsumerWarps * 16 * NT * 8;                       // [16][Bl]
    float* xinv = fin + 16 * p.sgrp;                                       // [Bl] 1/scale of each sequence
    uint64_t* full = reinterpret_cast<uint64_t*>(xinv + NT * 8 + 2);  // 8-byte aligned
    uint64_t* empty = full + p.stages;
    uint64_t* xbar = empty + p.stages;                                // the activation copy
    int* ticket = reinterpret_cast<int*>(xbar + 1);

    const int k_split = blockIdx.x % p.nk;
    const int cta_per_k = gridDim.x / p.nk;
    const int t_first = blockIdx.x / p.nk;
    const int b_lo = k_split * p.kr;
    const int b_hi = min(p.nb, b_lo + p.kr);
    const int nblk = max(0, b_hi - b_lo);
    const int stages_per_tile = (nblk + p.kb - 1) / p.kb;

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.stages; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, kConsumerWarps); }
        mbar_init(xbar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer: stream this CTA's tile-blocks ----------------
        if (lane == 0 && nblk > 0) {
            // The weights do not depend on the previous kernel: fill the ring
            // first, then wait for the activations (programmatic dependency)
            // before the first blocking wait on a ring slot.
            bool x_issued = false;
            auto issue_x = [&]() {
                // one group: the split's records are contiguous, one bulk copy; several
                // groups: the consumers gather their slice with cp.async instead
                if (Bl == B) {
                    pdl_wait();
                    mbar_expect_tx(xbar, (uint32_t)nblk * B * 128);
                    bulk_g2s(xs, p.xg + rec_off(b_lo, 0, B, 0, 0), (uint32_t)nblk * B * 128, xbar);
                }
                x_issued = true;
            };
            int it = 0;
            bool ok = true;
            for (int t = t_first; t < p.ntiles && ok; t += cta_per_k) {
                for (int st = 0; st < stages_per_tile; ++st, ++it) {
                    const int slot = it % p.stages;
                    const uint32_t ph = (uint32_t)(it / p.stages) & 1u;
                    if (!x_issued && it >= p.stages) issue_x();
                    if (!mbar_wait(empty + slot, ph ^ 1u, p.err)) { ok = false; break; }
                    const int b0 = b_lo + st * p.kb;
                    const int n = min(p.kb, b_hi - b0);
                    uint8_t* dst = ring + slot * stage_bytes;
                    const size_t tb = (size_t)t * p.nb + b0;
                    mbar_expect_tx(full + slot, (uint32_t)(n * (QB + SB)));
                    bulk_g2s(dst, p.q + tb * QB, (uint32_t)(n * QB), full + slot);
                    if (SB) bulk_g2s(dst + p.kb * QB, p.s + tb * SB, (uint32_t)(n * SB), full + slot);
                }
            }
            if (!x_issued) issue_x();
            // leave only after every copy issued into this CTA's shared memory has landed
            const int issued = it;
            for (int j = max(0, issued - p.stages); j < issued; ++j)
                mbar_wait(full + (j % p.stages), (uint32_t)(j / p.stages) & 1u, p.err);
            if (Bl == B) mbar_wait(xbar, 0u, p.err);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int ctid = threadIdx.x;  // 0 .. 255
    constexpr int NC = kConsumerWarps * 32;
    pdl_wait();

    // activations of this K split: the producer's bulk copy of the prepared
    // records (or this group's slice, gathered here), plus the split's scale per sequence
    bool aborted = false;
    if (nblk > 0 && Bl != B) load_rec_slice(xs, p.xg, b_lo, nblk, B, s0, Bl, ctid, NC);  // in flight meanwhile
    seq_scales(p, k_split, s0, Bl, xinv, ctid, NC);
    if (nblk > 0) {
        if (Bl == B) aborted = !mbar_wait(xbar, 0u, p.err);
        else cp_async_wait_all();
    }
    named_sync(1, NC);
    pdl_launch_dependents();

    int it = 0;  // `aborted`: a wait ran out: keep the barrier protocol, skip the math
    for (int t = t_first; t < p.ntiles; t += cta_per_k) {
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

        for (int st = 0; st < stages_per_tile; ++st, ++it) {
            const int slot = it % p.stages;
            if (!aborted && !mbar_wait(full + slot, (uint32_t)(it / p.stages) & 1u, p.err)) aborted = true;
            const uint8_t* sq = ring + slot * stage_bytes;
            const uint8_t* ss = sq + p.kb * QB;
            const int n = aborted ? 0 : min(p.kb, b_hi - (b_lo + st * p.kb));
            for (int bi = warp; bi < n; bi += kConsumerWarps) {
                const int bl = st * p.kb + bi;  // block index within the split
                uint32_t ra[4], rb[4];          // rows g and g+8, four half2 each
                if (WT == T_Q4_0) {
                    const uint2 w = *reinterpret_cast<const uint2*>(sq + bi * QB + lane * 8);
                    decode_q4(w.x, ra);
                    decode_q4(w.y, rb);
                } else if (WT == T_Q8_0) {
                    const uint4 w = *reinterpret_cast<const uint4*>(sq + bi * QB + lane * 16);
                    decode_q8(w.x, w.y, ra);
                    decode_q8(w.z, w.w, rb);
                } else {
                    const uint4 w0 = *reinterpret_cast<const uint4*>(sq + bi * QB + lane * 32);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(sq + bi * QB + lane * 32 + 16);
                    ra[0] = w0.x; ra[1] = w0.y; ra[2] = w0.z; ra[3] = w0.w;
                    rb[0] = w1.x; rb[1] = w1.y; rb[2] = w1.z; rb[3] = w1.w;
                }
                float dg = 1.f, dg8 = 1.f;
                if (WT != T_F16) {
                    const uint32_t dp = *reinterpret_cast<const uint32_t*>(ss + bi * SB + g * 4);
                    const float2 df = __half22float2(*reinterpret_cast<const __half2*>(&dp));
                    dg = df.x; dg8 = df.y;
                }
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const int s = j * 8 + g;
                    uint4 xh = make_uint4(0, 0, 0, 0), xl = make_uint4(0, 0, 0, 0);
                    if (s < Bl) {
                        xh = *reinterpret_cast<const uint4*>(xs + rec_off(bl, 0, Bl, s, c));
                        xl = *reinterpret_cast<const uint4*>(xs + rec_off(bl, 1, Bl, s, c));
                    }
                    if (WT == T_F16) {
                        mma16816(acc[j], ra[0], rb[0], ra[1], rb[1], xh.x, xh.y);
                        mma16816(acc[j], ra[0], rb[0], ra[1], rb[1], xl.x, xl.y);
                        mma16816(acc[j], ra[2], rb[2], ra[3], rb[3], xh.z, xh.w);
                        mma16816(acc[j], ra[2], rb[2], ra[3], rb[3], xl.z, xl.w);
                    } else {
                        float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
                        mma16816(t0, ra[0], rb[0], ra[1], rb[1], xh.x, xh.y);
                        mma16816(t1, ra[2], rb[2], ra[3], rb[3], xh.z, xh.w);
                        mma16816(t0, ra[0], rb[0], ra[1], rb[1], xl.x, xl.y);
                        mma16816(t1, ra[2], rb[2], ra[3], rb[3], xl.z, xl.w);
                        acc[j][0] = fmaf(dg, t0[0] + t1[0], acc[j][0]);
                        acc[j][1] = fmaf(dg, t0[1] + t1[1], acc[j][1]);
                        acc[j][2] = fmaf(dg8, t0[2] + t1[2], acc[j][2]);
                        acc[j][3] = fmaf(dg8, t0[3] + t1[3], acc[j][3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + slot);
        }

        // ---- reduce the 8 consumer warps: red[w][row][n]
        float* rw = red + warp * 16 * NT * 8;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            rw[g * NT * 8 + j * 8 + 2 * c] = acc[j][0];
            rw[g * NT * 8 + j * 8 + 2 * c + 1] = acc[j][1];
            rw[(g + 8) * NT * 8 + j * 8 + 2 * c] = acc[j][2];
            rw[(g + 8) * NT * 8 + j * 8 + 2 * c + 1] = acc[j][3];
        }
        named_sync(1, NC);
        for (int i = ctid; i < 16 * Bl; i += NC) {
            const int r = i / Bl, s = i % Bl;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) v += red[w * 16 * NT * 8 + r * NT * 8 + s];
            fin[r * Bl + s] = v * xinv[s];
        }
        named_sync(1, NC);

        // ---- split-K: the last CTA of this (row tile, group) adds the partials in split order
        if (p.nk > 1) {
            float* pt = p.part + (size_t)t * p.nk * 16 * B;  // [nk][16][B]
            for (int i = ctid; i < 16 * Bl; i += NC)
                pt[(size_t)k_split * 16 * B + (i / Bl) * B + s0 + i % Bl] = fin[i];
            __threadfence();
            named_sync(1, NC);
            unsigned* cnt = p.tile_cnt + (size_t)t * gridDim.y + blockIdx.y;
            if (ctid == 0) *ticket = (int)atomicAdd(cnt, 1u) == p.nk - 1;
            named_sync(1, NC);
            if (!*ticket) continue;
            __threadfence();
            for (int i = ctid; i < 16 * Bl; i += NC) {
                const size_t gi = (size_t)(i / Bl) * B + s0 + i % Bl;
                float v = 0.f;
                for (int k = 0; k < p.nk; ++k) v += __ldcg(pt + (size_t)k * 16 * B + gi);
                fin[i] = v;
            }
            if (ctid == 0) *cnt = 0u;
            named_sync(1, NC);
        }

        // ---- epilogue on fin[16][B]
        const int r0 = t * 16;
        if ((EPI == EPI_ADD || EPI == EPI_SWIGLU) && p.rec_out) {
            // the tile's outputs and their records for the next projection, one element per
            // thread (consecutive threads: consecutive rows of one sequence); then (residual)
            // the tile's sum of squares per sequence, in row order, from the new values in fin
            const int rows_here = min(16, p.rows - r0);
            if (EPI == EPI_ADD) {
                for (int i = ctid; i < 16 * Bl; i += NC) {
                    const int rl = i & 15, s = i >> 4, r = r0 + rl;
                    if (rl >= rows_here) continue;
                    float* o = p.out + (size_t)(s0 + s) * p.ldo + r;
                    const float xn = *o + fin[rl * Bl + s];
                    *o = xn;
                    fin[rl * Bl + s] = xn;
                    store_act_record(p.rec_out, B, r, s0 + s, p.rec_w ? xn * p.rec_w[r] : xn);
                }
                if (p.ss_out) {
                    named_sync(1, NC);
                    for (int s = ctid; s < Bl; s += NC) {
                        float ssum = 0.f;
                        for (int rl = 0; rl < rows_here; ++rl) ssum = fmaf(fin[rl * Bl + s], fin[rl * Bl + s], ssum);
                        p.ss_out[(size_t)t * B + s0 + s] = ssum;
                    }
                }
            } else {
                for (int i = ctid; i < 8 * Bl; i += NC) {
                    const int rp = i & 7, s = i >> 3, rl = 2 * rp, r = r0 + rl;
                    if (rl >= rows_here) continue;
                    const float val = fin[rl * Bl + s], up = fin[(rl + 1) * Bl + s];
                    const float a = (val / (1.f + expf(-val))) * up;
                    p.out[(size_t)(s0 + s) * p.ldo + (r >> 1)] = a;
                    store_act_record(p.rec_out, B, r >> 1, s0 + s, a);
                }
            }
            named_sync(1, NC);  // fin/red reused by the next tile
            continue;
        }
        for (int i = ctid; i < 16 * Bl; i += NC) {
            const int rl = i / Bl, sl = i % Bl, r = r0 + rl, s = s0 + sl;
            if (r >= p.rows) continue;
            const float val = fin[i];
            if (EPI == EPI_STORE) {
                p.out[(size_t)s * p.ldo + r] = val;
            } else if (EPI == EPI_ADD) {
                p.out[(size_t)s * p.ldo + r] += val;
            } else if (EPI == EPI_SWIGLU) {
                // row 2o = gate o, row 2o+1 = up o: out[o] = silu(gate) * up
                if ((rl & 1) == 0) {
                    const float up = fin[(rl + 1) * Bl + sl];
                    p.out[(size_t)s * p.ldo + (r >> 1)] = (val / (1.f + expf(-val))) * up;
                }
            } else {  // EPI_QKV
                const int slot = p.slots[s], ps = p.pos[slot];
                int rr = r, region = 0;  // 0 q, 1 k, 2 v
                if (rr >= p.q_rows) { rr -= p.q_rows; region = 1; if (rr >= p.kv_rows) { rr -= p.kv_rows; region = 2; } }
                const int d = rr % p.head_dim;
                float o = val;
                if (region < 2 && d < 2 * p.rope_pairs) {
                    const float2 cs = p.rope_cs[(size_t)ps * p.rope_pairs + (d >> 1)];
                    const float other = fin[(rl ^ 1) * Bl + sl];
                    // adjacent-pair rotation, unfused to keep the reference's rounding
                    if ((d & 1) == 0) o = __fsub_rn(__fmul_rn(val, cs.x), __fmul_rn(other, cs.y));
                    else o = __fadd_rn(__fmul_rn(other, cs.y), __fmul_rn(val, cs.x));
                }
                if (region == 0) {
                    p.out[(size_t)s * p.ldo + rr] = o;
                } else {
                    KV* base = reinterpret_cast<KV*>(region == 1 ? p.kc : p.vc);
                    base[(size_t)slot * p.kv_slot_stride + ((size_t)(rr / p.head_dim) * p.kv_cap + ps) * p.head_dim + d] =
                        kv_from<KV>(o);
                }
            }
        }
        named_sync(1, NC);  // fin/red reused by the next tile
    }
}

// ---------------------------------------------------------------------------
// the wide kernel: y = W x with EPI_STORE for matrices of many row tiles and a
// short K (the lm_head of a small model). Each consumer warp owns whole row
// tiles -- all K blocks of a tile in one ring stage, no cross-warp reduction
// and no CTA barrier per tile -- so the warps stream independently. Stage i of
// the ring belongs to warp i % 8 (stages: a multiple of 8); the producer fills
// the stages in tile order. Grid (CTAs, sequence groups) like the tile kernel;
// tiles t = blockIdx.x + i * gridDim.x. Shared memory:
//   ring [stages][nb * (QB + SB)] | xs: records of nb blocks x sgrp | xinv [sgrp] | barriers
// ---------------------------------------------------------------------------
__host__ __device__ constexpr size_t mv_wide_smem(int type, int nb, int sgrp, int stages) {
    return (size_t)stages * nb * (tile_qbytes(type) + (type == T_F16 ? 0 : kTileSBytes)) + (size_t)nb * sgrp * 128 +
           (size_t)sgrp * 4 + 16 + (size_t)(2 * stages + 1) * 8;
}

template <int WT, int NT>
__global__ void __launch_bounds__(kMvThreads, 1) mv_wide_kernel(const MvParams p) {
    constexpr int QB = tile_qbytes(WT);
    constexpr int SB = WT == T_F16 ? 0 : kTileSBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int B = p.nseq;
    const int s0 = blockIdx.y * p.sgrp;
    const int Bl = min(p.sgrp, B - s0);
    const int nb = p.nb;
    const int tile_bytes = nb * (QB + SB);
    const int S = p.stages;

    uint8_t* ring = smem;
    uint8_t* xs = ring + (size_t)S * tile_bytes;                        // records of [nb] blocks x [Bl]
    float* xinv = reinterpret_cast<float*>(xs + (size_t)nb * p.sgrp * 128);
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(xinv + p.sgrp) + 15) & ~uintptr_t(15));
    uint64_t* empty = full + S;
    uint64_t* xbar = empty + S;

    const int n_local = blockIdx.x < p.ntiles ? (p.ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, 1); }
        mbar_init(xbar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0 && n_local > 0) {
            bool x_issued = false;
            auto issue_x = [&]() {  // several groups: the consumers gather their slice
                if (Bl == B) {
                    pdl_wait();
                    mbar_expect_tx(xbar, (uint32_t)nb * B * 128);
                    bulk_g2s(xs, p.xg, (uint32_t)nb * B * 128, xbar);
                }
                x_issued = true;
            };
            int i = 0;
            for (; i < n_local; ++i) {
                const int slot = i % S;
                if (!x_issued && i >= S) issue_x();
                if (!mbar_wait(empty + slot, ((uint32_t)(i / S) & 1u) ^ 1u, p.err)) break;
                const size_t t = (size_t)blockIdx.x + (size_t)i * gridDim.x;
                uint8_t* dst = ring + (size_t)slot * tile_bytes;
                mbar_expect_tx(full + slot, (uint32_t)tile_bytes);
                bulk_g2s(dst, p.q + t * nb * QB, (uint32_t)(nb * QB), full + slot);
                if (SB) bulk_g2s(dst + nb * QB, p.s + t * nb * SB, (uint32_t)(nb * SB), full + slot);
            }
            if (!x_issued) issue_x();
            for (int j = max(0, i - S); j < i; ++j) mbar_wait(full + (j % S), (uint32_t)(j / S) & 1u, p.err);
            if (Bl == B) mbar_wait(xbar, 0u, p.err);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int ctid = threadIdx.x;
    constexpr int NC = kConsumerWarps * 32;
    pdl_wait();
    bool aborted = false;
    if (n_local > 0 && Bl != B) load_rec_slice(xs, p.xg, 0, nb, B, s0, Bl, ctid, NC);  // in flight meanwhile
    seq_scales(p, 0, s0, Bl, xinv, ctid, NC);
    if (n_local > 0) {
        if (Bl == B) aborted = !mbar_wait(xbar, 0u, p.err);
        else cp_async_wait_all();
    }
    named_sync(1, NC);
    pdl_launch_dependents();

    for (int i = warp; i < n_local; i += kConsumerWarps) {
        const int slot = i % S;
        if (!aborted && !mbar_wait(full + slot, (uint32_t)(i / S) & 1u, p.err)) aborted = true;
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        const uint8_t* sq = ring + (size_t)slot * tile_bytes;
        const uint8_t* ss = sq + nb * QB;
        for (int bl = 0; bl < (aborted ? 0 : nb); ++bl) {
            uint32_t ra[4], rb[4];
            if (WT == T_Q4_0) {
                const uint2 w = *reinterpret_cast<const uint2*>(sq + bl * QB + lane * 8);
                decode_q4(w.x, ra);
                decode_q4(w.y, rb);
            } else if (WT == T_Q8_0) {
                const uint4 w = *reinterpret_cast<const uint4*>(sq + bl * QB + lane * 16);
                decode_q8(w.x, w.y, ra);
                decode_q8(w.z, w.w, rb);
            } else {
                const uint4 w0 = *reinterpret_cast<const uint4*>(sq + bl * QB + lane * 32);
                const uint4 w1 = *reinterpret_cast<const uint4*>(sq + bl * QB + lane * 32 + 16);
                ra[0] = w0.x; ra[1] = w0.y; ra[2] = w0.z; ra[3] = w0.w;
                rb[0] = w1.x; rb[1] = w1.y; rb[2] = w1.z; rb[3] = w1.w;
            }
            float dg = 1.f, dg8 = 1.f;
            if (WT != T_F16) {
                const uint32_t dp = *reinterpret_cast<const uint32_t*>(ss + bl * SB + g * 4);
                const float2 df = __half22float2(*reinterpret_cast<const __half2*>(&dp));
                dg = df.x; dg8 = df.y;
            }
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int s = j * 8 + g;
                uint4 xh = make_uint4(0, 0, 0, 0), xl = make_uint4(0, 0, 0, 0);
                if (s < Bl) {
                    xh = *reinterpret_cast<const uint4*>(xs + rec_off(bl, 0, Bl, s, c));
                    xl = *reinterpret_cast<const uint4*>(xs + rec_off(bl, 1, Bl, s, c));
                }
                if (WT == T_F16) {
                    mma16816(acc[j], ra[0], rb[0], ra[1], rb[1], xh.x, xh.y);
                    mma16816(acc[j], ra[0], rb[0], ra[1], rb[1], xl.x, xl.y);
                    mma16816(acc[j], ra[2], rb[2], ra[3], rb[3], xh.z, xh.w);
                    mma16816(acc[j], ra[2], rb[2], ra[3], rb[3], xl.z, xl.w);
                } else {
                    // two independent chains (columns 0-15 and 16-31 of the block)
                    float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(t0, ra[0], rb[0], ra[1], rb[1], xh.x, xh.y);
                    mma16816(t1, ra[2], rb[2], ra[3], rb[3], xh.z, xh.w);
                    mma16816(t0, ra[0], rb[0], ra[1], rb[1], xl.x, xl.y);
                    mma16816(t1, ra[2], rb[2], ra[3], rb[3], xl.z, xl.w);
                    acc[j][0] = fmaf(dg, t0[0] + t1[0], acc[j][0]);
                    acc[j][1] = fmaf(dg, t0[1] + t1[1], acc[j][1]);
                    acc[j][2] = fmaf(dg8, t0[2] + t1[2], acc[j][2]);
                    acc[j][3] = fmaf(dg8, t0[3] + t1[3], acc[j][3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
        if (aborted) continue;
        // rows g and g + 8 of the tile, sequences j * 8 + 2c and + 1
        const int r = (blockIdx.x + i * gridDim.x) * 16 + g;
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int s = j * 8 + 2 * c + (e & 1), rr = r + (e >> 1) * 8;
                if (s < Bl && rr < p.rows) p.out[(size_t)(s0 + s) * p.ldo + rr] = acc[j][e] * xinv[s];
            }
    }
}

// ---------------------------------------------------------------------------
// activation preparation: grid (nk, nseq), one CTA per (K split, sequence)
// ---------------------------------------------------------------------------
// rmsnorm (when norm_w is set) of the sequence's row, a power-of-two scale
// per K split that puts the split's max |x| into [2^10, 2^11), and the scaled
// values as binary16 hi + lo in the tile kernel's fragment order.
constexpr int kXPrepThreads = 256;

static __global__ void __launch_bounds__(kXPrepThreads) xprep_kernel(const XPrepParams p) {
    __shared__ float red[kXPrepThreads / 32][2];
    __shared__ float stat[2];
    pdl_launch_dependents();  // the matvec may start streaming its weights
    pdl_wait();
    const int k = blockIdx.x, s = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int b_lo = k * p.kr, b_hi = min(p.nb, b_lo + p.kr);
    const int nv = p.in >> 2, v_lo = b_lo * 8, v_hi = b_hi * 8;  // float4 indices
    const float4* x4 = reinterpret_cast<const float4*>(p.x + (size_t)s * p.ldx);
    const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
    float ss = 0.f, mx = 0.f;
    if (p.norm_w) {
        for (int f = threadIdx.x; f < nv; f += kXPrepThreads) {
            const float4 v = x4[f];
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
            if (f >= v_lo && f < v_hi) {
                const float4 w = w4[f];
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * w.x), fabsf(v.y * w.y)), fmaxf(fabsf(v.z * w.z), fabsf(v.w * w.w))));
            }
        }
    } else {
        for (int f = v_lo + threadIdx.x; f < v_hi; f += kXPrepThreads) {
            const float4 v = x4[f];
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if (lane == 0) { red[warp][0] = ss; red[warp][1] = mx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f, m = 0.f;
        for (int w = 0; w < kXPrepThreads / 32; ++w) { a += red[w][0]; m = fmaxf(m, red[w][1]); }
        const float iv = p.norm_w ? 1.f / sqrtf(a / float(p.in) + p.eps) : 1.f;
        m *= iv;
        int ex = 0;
        if (m > 0.f && isfinite(m)) { frexpf(m, &ex); ex = max(-100, min(100, ex)); }
        const float xi = ldexpf(1.f, ex - 11);
        stat[0] = iv;
        stat[1] = xi;
        p.xinv[(size_t)k * p.nseq + s] = xi;
    }
    __syncthreads();
    const float iv = stat[0], up = 1.f / stat[1];  // exact: a power of two
    // one 8-element group (one lane's fragment record) per thread
    const int ng = (b_hi - b_lo) * 4;
    for (int gi = threadIdx.x; gi < ng; gi += kXPrepThreads) {
        const int f = v_lo + 2 * gi;
        const float4 a0 = x4[f], a1 = x4[f + 1];
        float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        if (p.norm_w) {
            const float4 c0 = w4[f], c1 = w4[f + 1];
            const float w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = v[e] * (iv * w[e]);
        }
        __align__(16) __half hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float u = v[e] * up;
            const __half h = __float2half_rn(u);
            hi[frag_pos(e)] = h;
            lo[frag_pos(e)] = __float2half_rn(u - __half2float(h));
        }
        const int bl = b_lo + (gi >> 2), c = gi & 3;
        *reinterpret_cast<uint4*>(p.xg + rec_off(bl, 0, p.nseq, s, c)) = *reinterpret_cast<const uint4*>(hi);
        *reinterpret_cast<uint4*>(p.xg + rec_off(bl, 1, p.nseq, s, c)) = *reinterpret_cast<const uint4*>(lo);
    }
}

}  // namespace laic
