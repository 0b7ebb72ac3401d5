// Team variant of the fragment-tile matvec for small batches (the decode
// latency path: one to a few sequences whose activations fit in shared memory).
//
// Each CTA owns a contiguous run of whole 16-row tiles. Its warps form teams
// of k warps; a team works on one tile at a time and warp i of the team takes
// the i-th contiguous slice of the tile's K range. Every warp streams its
// slices through its own shared-memory ring with 1-D bulk TMA copies issued by
// its lane 0 (the first stages go out before the programmatic-dependent-launch
// wait: weights never depend on the previous kernel), decodes and multiplies
// with mma.sync like mv_mma_kernel, then drops its 16 x B partial sums into a
// per-warp shared-memory slot and takes a shared-memory ticket. The warp that
// completes a tile adds the team's partials in warp order (deterministic) and
// runs the epilogue. The streaming loop never waits on global memory, and no
// CTA-wide barrier is taken after the activation prologue.
//
// NT = 0 is the single-sequence integer variant for Q4_0 / Q8_0: the same
// tiles and rings, but exact integer dot products of the quants with the
// activation split into three int8 digits, on the integer tensor-core path
// (mma.m16n8k32, u8 x s8 or s8 x s8 -> s32), instead of converting quants to
// binary16, where one sequence fills 2 of the 8 product columns. Per 32-column
// block the activation is scaled by a power of two that puts its largest
// magnitude in [2^19, 2^20), rounded to an integer x (21 bits, exact in the
// digits below) and written as balanced base-128 digits
// x = p0 * 2^14 + p1 * 2^7 + p2 (each in [-64, 64]). The digits are the first
// three columns of the product's B operand, so one mma gives, per row of the
// 16-row tile-block,
//   sum_k q_k x_k = 2^14 sum q p0 + 2^7 sum q p1 + sum q p2
// with q the stored quant (Q4_0: the nibble n, corrected by -8 * sum x; Q8_0:
// the int8 value), all in int32 without rounding; then
//   acc += float(sum) * d * 2^-scale   (d the block scale, FP32 accumulate).
#pragma once
#include "mma_matvec.cuh"

namespace laic {

// Launch shape (overridable at build time for tuning sweeps).
#ifndef LAIC_SK_WARPS
#define LAIC_SK_WARPS 16
#endif
#ifndef LAIC_SK_RING_BYTES
#define LAIC_SK_RING_BYTES 4608
#endif
#ifndef LAIC_SK_STAGE_BYTES
#define LAIC_SK_STAGE_BYTES 2304
#endif
constexpr int kSkWarps = LAIC_SK_WARPS;          // warps per CTA
constexpr int kSkRingBytes = LAIC_SK_RING_BYTES;  // per warp: stages in flight
constexpr int kSkSlots = 2;                       // tile slots per team (a team's warps may drift apart)
// largest power of two dividing the warp count: the widest team
// Large one-sequence matrices (at least 128 blocks per row and 4096 rows) run with more warps
// per CTA: more weight stages in flight and more warps to hide the integer loop's latencies
// (measured: the 8B-shaped step 8 % faster; 1B-shaped projections ~4 % slower, so they keep 16).
constexpr int kSkWarpsWide = 24;
__host__ __device__ constexpr int sk_max_team(int w) { return (w & -w) < 16 ? (w & -w) : 16; }
// tile-blocks per ring stage (about LAIC_SK_STAGE_BYTES for every type)
__host__ __device__ constexpr int sk_kb(int type) {
    return LAIC_SK_STAGE_BYTES / (tile_qbytes(type) + (type == T_F16 ? 0 : kTileSBytes)) > 0
               ? LAIC_SK_STAGE_BYTES / (tile_qbytes(type) + (type == T_F16 ? 0 : kTileSBytes)) : 1;
}
__host__ __device__ constexpr int sk_stage_bytes(int type) {
    return sk_kb(type) * (tile_qbytes(type) + (type == T_F16 ? 0 : kTileSBytes));
}
__host__ __device__ constexpr int sk_stages(int type) { return kSkRingBytes / sk_stage_bytes(type); }
// warps per tile: long rows are split over more warps
__host__ __device__ inline int sk_team(int nb, int w = kSkWarps) {
    const int k = nb >= 256 ? 16 : nb >= 128 ? 8 : nb >= 64 ? 4 : nb >= 32 ? 2 : 1;
    return k < sk_max_team(w) ? k : sk_max_team(w);
}
// Rough cost of one warp's work with teams of k warps, in eighths of a tile-block: the
// rounds of tiles its team takes (a CTA owns ceil(ntiles / grid) whole tiles), each a
// slice of ceil(nb / k) blocks plus the team's merge (about k / 8 blocks).
__host__ __device__ inline int sk_team_cost(int k, int nb, int ntiles, int grid, int w) {
    const int tpc = (ntiles + grid - 1) / grid, teams = w / k;
    return (tpc + teams - 1) / teams * (8 * ((nb + k - 1) / k) + k);
}
// Team size of a launch: sk_team, or a larger divisor of w that cuts the cost by more
// than 10 % (few tiles per CTA leave teams idle: the 4096-row projections of an 8B-shaped
// model own one or two tiles per CTA), keeping at least two blocks per warp. Rows of more
// than 256 blocks keep sk_team: their slices are long already (measured: 12-warp teams
// on 448-block rows were 6 % slower than 8-warp teams).
__host__ __device__ inline int sk_team_for(int nb, int ntiles, int grid, int w) {
    int k = sk_team(nb, w);
    if (nb > 256) return k;
    int best = sk_team_cost(k, nb, ntiles, grid, w);
    for (int kk = k + 1; kk <= w; ++kk) {
        if (w % kk != 0 || 2 * kk > nb) continue;
        const int c = sk_team_cost(kk, nb, ntiles, grid, w);
        if (10 * c < 9 * best) { best = c; k = kk; }
    }
    return k;
}
// The team kernel's split of a launch (grid CTAs of w warps) into MvParams: teams of
// sk_team_for warps, whole tiles per CTA, equal K slices per warp of a team.
inline void sk_split(MvParams& p, int grid, int w) {
    const int k = sk_team_for(p.nb, p.ntiles, grid, w);
    p.team_k = k;
    p.team_n = w / k;
    p.team_inv = (65536 + k - 1) / k;  // exact for warp indices below 64
    p.tq = p.ntiles / grid;
    p.tr = p.ntiles % grid;
    p.sq = p.nb / k;
    p.sr = p.nb % k;
}

// One warp's share of a team-kernel launch, from sk_split's parameters: its team, its place in the
// team and the team's first warp, the CTA's row tiles [t_lo, t_hi) (the team takes t_lo + team,
// + teams, ...) and the warp's K slice [b_lo, b_hi) of every tile. Shared by the kernel and the
// host-side check of the split.
struct SkWarpRange {
    int team, wi, leader, t_lo, t_hi, b_lo, b_hi;
};
__host__ __device__ inline SkWarpRange sk_warp_range(const MvParams& p, int cta, int warp) {
    SkWarpRange r;
    r.team = (warp * p.team_inv) >> 16;
    r.wi = warp - r.team * p.team_k;
    r.leader = r.team * p.team_k;
    r.t_lo = cta * p.tq + (cta < p.tr ? cta : p.tr);
    r.t_hi = r.t_lo + p.tq + (cta < p.tr ? 1 : 0);
    r.b_lo = r.wi * p.sq + (r.wi < p.sr ? r.wi : p.sr);
    r.b_hi = r.b_lo + p.sq + (r.wi < p.sr ? 1 : 0);
    return r;
}

// tickets, merged-tile marks, per-warp statistics, 1/rms and split scale per sequence
__host__ __device__ inline size_t sk_small_bytes(int B, int w = kSkWarps) {
    return ((size_t)w * kSkSlots * 2 * 4 + (size_t)w * B * 2 * 4 + 2 * (size_t)B * 4 + 15) / 16 * 16;
}
// Shared memory of one CTA: rings, activations (whole K), partial slots + tickets, statistics, barriers.
__host__ __device__ inline size_t sk_smem_bytes(int type, int nb, int B, int w = kSkWarps) {
    const size_t rings = (size_t)w * sk_stages(type) * sk_stage_bytes(type);
    const size_t xs = (size_t)nb * B * 128;
    const size_t parts = (size_t)w * kSkSlots * 16 * B * 4;  // [warp][slot][16][B]
    return rings + xs + parts + sk_small_bytes(B, w) + (size_t)w * sk_stages(type) * 8;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// d = sum of the four products of unsigned bytes of a and signed bytes of b, plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Activation record of one 32-column block for the team kernel's integer variant,
// laid out as the B operand of mma.m16n8k32 (column n = digit, k = the 32 columns
// in the quants' fragment order): at d * 32 + c * 8 the two words of digit d (p0,
// p1, p2) over 8-column group c (the bytes in the order of the quants of group c
// in a lane's fragment, dp_byte_of), then at 96 the int -8 * sum x over the block
// (Q4_0, else 0) and the block's scale 2^-s as a float; 24 bytes of padding.
constexpr int kDpRecBytes = 128;
// The decode-step kernel's records (dp_lane_record) keep one scale per 8-column
// group instead: for each group c, 32 bytes at c * 32 with digits p0, p1, p2 as
// two words each, then -8 * sum x over the group (Q4_0, else 0) and the group's
// scale 2^-s as a float.

// Byte of element k (0..7) of an 8-column group inside the two words of a
// lane's fragment: Q4_0 packs (e0,e1) (e2,e3) (e4,e5) (e6,e7) as nibble pairs,
// read as low nibbles (e0 e2 e4 e6) and high nibbles (e1 e3 e5 e7);
// Q8_0 stores e0 e4 e1 e5 | e2 e6 e3 e7.
template <int WT>
__device__ __forceinline__ int dp_byte_of(int k) {
    if (WT == T_Q4_0) return (k & 1) * 4 + (k >> 1);
    return frag_pos(k);
}

// A phase of the decode-step kernel makes the records of the values it writes for
// its next projection (one scale per 8-column group, the step kernel's layout), one
// 8-column group per 8 lanes: `val` is this lane's value (0 where none), `k` its
// index in the group and `gidx` the group (negative: no record); every lane of the
// warp must call it. Returns the group's sum of `sq` (for the next rmsnorm), valid
// in the group's lane k = 0.
template <int WT>
__device__ __forceinline__ float dp_lane_record(float val, float sq, int k, int gidx, uint8_t* recs, int m1, int m2,
                                                   int m3) {
    float mx = fabsf(val);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m3));
    int ex = 0;
    if (mx > 0.f && isfinite(mx)) frexpf(mx, &ex);
    const int xi = (int)rintf(ldexpf(val, 20 - ex));
    const int p2 = ((xi + 64) & 127) - 64;
    const int t1 = (xi - p2) >> 7;
    const int p1 = ((t1 + 64) & 127) - 64;
    const int p0 = (t1 - p1) >> 7;
    int gs = xi;
    gs += __shfl_xor_sync(0xffffffffu, gs, m1);
    gs += __shfl_xor_sync(0xffffffffu, gs, m2);
    gs += __shfl_xor_sync(0xffffffffu, gs, m3);
    sq += __shfl_xor_sync(0xffffffffu, sq, m1);
    sq += __shfl_xor_sync(0xffffffffu, sq, m2);
    sq += __shfl_xor_sync(0xffffffffu, sq, m3);
    if (gidx >= 0) {
        uint8_t* rec = recs + (size_t)gidx * 32;
        const int pos = dp_byte_of<WT>(k);
        rec[pos] = (uint8_t)(int8_t)p0;
        rec[8 + pos] = (uint8_t)(int8_t)p1;
        rec[16 + pos] = (uint8_t)(int8_t)p2;
        if (k == 0) {
            reinterpret_cast<int*>(rec)[6] = WT == T_Q4_0 ? -8 * gs : 0;
            reinterpret_cast<float*>(rec)[7] = ldexpf(1.f, ex - 20);
        }
    }
    return sq;
}

// d = A (16x32, unsigned or signed bytes) x B (32x8, signed bytes) + c, in int32 (mma.m16n8k32)
template <bool AU8>
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    if constexpr (AU8)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
    else
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Per-lane constants of the integer variant. The product's columns 0, 1, 2 are the digit
// sums of rows g and g+8 (lane c holds columns 2c and 2c+1; lanes g = 3..7 load digit
// g mod 3, so columns 3..7 repeat them and are ignored): lane c = 0 forms
// 2^14 s0 + 2^7 s1, lane c = 1 forms s2 plus the block's -8 sum x, lanes c = 2, 3 nothing.
struct DpLane {
    int ka, kb, kx;       // weights of columns 2c, 2c+1 and of the block's correction (0 / -1 mask)
    uint32_t boff;        // this lane's B fragment in a record: digit g mod 3, group c
};
__device__ __forceinline__ DpLane dp_lane(int lane) {
    const int g = lane >> 2, c = lane & 3;
    DpLane l;
    l.ka = c == 0 ? 16384 : c == 1 ? 1 : 0;
    l.kb = c == 0 ? 128 : 0;
    l.kx = c == 1 ? -1 : 0;
    l.boff = (uint32_t)((g % 3) * 32 + c * 8);
    return l;
}

// One 16x32 tile-block of the integer variant: rows g and g+8 of this lane's share of the
// sum (added over the row's four lanes at the end of the tile).
template <int WT>
__device__ __forceinline__ void tile_block_dp(uint32_t q, uint32_t sc, uint32_t xrec, const DpLane& ln, int lane,
                                              float (&acc)[2]) {
    const int g = lane >> 2;
    const uint2 b = lds64(xrec + ln.boff);
    const uint2 xs = lds64(xrec + 96);  // -8 sum x, 2^-s
    const uint32_t dp = lds32(sc + g * 4);
    const float2 df = __half22float2(*reinterpret_cast<const __half2*>(&dp));
    int r[4];
    if (WT == T_Q4_0) {
        // A fragment: row g / g+8, k = 4c..4c+3 the low nibbles, k = 16+4c.. the high nibbles
        const uint2 w = lds64(q + lane * 8);
        imma16832<true>(r, w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, (w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu,
                        b.x, b.y);
    } else {
        const uint4 w = lds128(q + lane * 16);
        imma16832<false>(r, w.x, w.z, w.y, w.w, b.x, b.y);
    }
    const int x8 = (int)xs.x & ln.kx;
    const float sinv = __uint_as_float(xs.y);
    const int v0 = r[0] * ln.ka + r[1] * ln.kb + x8;  // exact: |v| < 2^30
    const int v1 = r[2] * ln.ka + r[3] * ln.kb + x8;
    acc[0] = fmaf((float)v0, df.x * sinv, acc[0]);
    acc[1] = fmaf((float)v1, df.y * sinv, acc[1]);
}

// One 16x32 tile-block: decode this lane's A fragments, multiply with the
// activation columns (hi and lo parts side by side) and add d * result.
// `xlane` points at this lane's activation record of block 0 (a padding column
// reuses the last real one); records of consecutive blocks are `xstride` apart.
template <int WT, int NT>
__device__ __forceinline__ void tile_block(uint32_t q, uint32_t sc, const uint32_t (&xlane)[NT], int b, int xstride,
                                           int lane, float (&acc)[NT][4]) {
    const int g = lane >> 2;
    uint32_t ra[4], rb[4];
    if (WT == T_Q4_0) {
        const uint2 w = lds64(q + lane * 8);
        decode_q4(w.x, ra);
        decode_q4(w.y, rb);
    } else if (WT == T_Q8_0) {
        const uint4 w = lds128(q + lane * 16);
        decode_q8(w.x, w.y, ra);
        decode_q8(w.z, w.w, rb);
    } else {
        const uint4 w0 = lds128(q + lane * 32);
        const uint4 w1 = lds128(q + lane * 32 + 16);
        ra[0] = w0.x; ra[1] = w0.y; ra[2] = w0.z; ra[3] = w0.w;
        rb[0] = w1.x; rb[1] = w1.y; rb[2] = w1.z; rb[3] = w1.w;
    }
    float dg = 1.f, dg8 = 1.f;
    if (WT != T_F16) {
        const uint32_t dp = lds32(sc + g * 4);
        const float2 df = __half22float2(*reinterpret_cast<const __half2*>(&dp));
        dg = df.x; dg8 = df.y;
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        // padding columns load a real record: their products land in output columns nobody reads
        const uint4 xv = lds128(xlane[j] + b * xstride);
        if (WT == T_F16) {
            mma16816_acc(acc[j], ra[0], rb[0], ra[1], rb[1], xv.x, xv.y);
            mma16816_acc(acc[j], ra[2], rb[2], ra[3], rb[3], xv.z, xv.w);
        } else {
            float t[4];
            mma16816_z(t, ra[0], rb[0], ra[1], rb[1], xv.x, xv.y);
            mma16816_acc(t, ra[2], rb[2], ra[3], rb[3], xv.z, xv.w);
            acc[j][0] = fmaf(dg, t[0], acc[j][0]);
            acc[j][1] = fmaf(dg, t[1], acc[j][1]);
            acc[j][2] = fmaf(dg8, t[2], acc[j][2]);
            acc[j][3] = fmaf(dg8, t[3], acc[j][3]);
        }
    }
}

// The digit record of one 8-column group of values v (thread-per-group, whole warp
// active, the four groups of a block in adjacent lanes): the block's power-of-two scale,
// the digits in the quants' byte order, and the record store (kDpRecBytes layout) when
// `live`. The block's exponent ex (its largest magnitude in [2^(ex-1), 2^ex)) comes from
// the float's bits and the scaling is one exact multiply by 2^(20-ex), rounded to nearest
// even as rintf(ldexpf(v, 20 - ex)) would; a block whose largest magnitude is below 2^-100,
// or not finite, is written as zeros.
template <int WT>
__device__ __forceinline__ void dp_group_digits(const float (&v)[8], int gi, bool live, uint8_t* xs) {
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) mx = fmaxf(mx, fabsf(v[k]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const int eb = (__float_as_int(mx) >> 23) & 0xFF;  // biased exponent (mx >= 0)
    const int ex = eb - 126;                             // mx in [2^(ex-1), 2^ex) for normal mx
    const bool ok = eb != 0xFF && ex > -100;
    const float sc = ok ? __int_as_float((147 - ex) << 23) : 0.f;  // 2^(20-ex), a normal float
    uint32_t dw[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};  // digit words p0 p1 p2, quant byte order
    int gs = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int xi = ok ? __float2int_rn(v[k] * sc) : 0;  // |xi| <= 2^20
        const int p2 = ((xi + 64) & 127) - 64;
        const int t1 = (xi - p2) >> 7;
        const int p1 = ((t1 + 64) & 127) - 64;
        const int p0 = (t1 - p1) >> 7;
        gs += xi;
        const int pos = dp_byte_of<WT>(k), wd = pos >> 2, sh = (pos & 3) * 8;
        dw[0][wd] |= (uint32_t)(p0 & 0xFF) << sh;
        dw[1][wd] |= (uint32_t)(p1 & 0xFF) << sh;
        dw[2][wd] |= (uint32_t)(p2 & 0xFF) << sh;
    }
    gs += __shfl_xor_sync(0xffffffffu, gs, 1);  // the block's sum over its four groups
    gs += __shfl_xor_sync(0xffffffffu, gs, 2);
    if (live) {
        uint8_t* rec = xs + (size_t)(gi >> 2) * kDpRecBytes;  // block gi/4, group gi%4
        const int c = gi & 3;
#pragma unroll
        for (int d = 0; d < 3; ++d) *reinterpret_cast<uint2*>(rec + d * 32 + c * 8) = make_uint2(dw[d][0], dw[d][1]);
        if (c == 0)
            *reinterpret_cast<uint2*>(rec + 96) = make_uint2((uint32_t)(WT == T_Q4_0 ? -8 * gs : 0),
                                                             ok ? (uint32_t)(107 + ex) << 23 : 0u);  // 2^(ex-20)
    }
}

// dp_group_digits of v scaled by iv * norm_w (when norm_w is given).
template <int WT>
__device__ __forceinline__ void dp_group_record(float (&v)[8], const float* norm_w, float iv, int gi, bool live,
                                                uint8_t* xs) {
    if (norm_w && live) {
        const float4 w0 = reinterpret_cast<const float4*>(norm_w)[2 * gi];
        const float4 w1 = reinterpret_cast<const float4*>(norm_w)[2 * gi + 1];
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = v[k] * (iv * w[k]);
    }
    dp_group_digits<WT>(v, gi, live, xs);
}

// Records of x * norm_w (norm_w may be null) for `nb` blocks, without the rmsnorm's 1/rms
// (whole CTA; ends with a CTA barrier): every thread loads its groups' activations and
// norm weights first (up to kDpGroupsInFlight groups per thread), then forms the digits.
constexpr int kDpGroupsInFlight = 3;
template <int WT>
__device__ __forceinline__ void dp_records_unscaled(const float* x, const float* norm_w, int nb, uint8_t* xs) {
    const int ng = nb * 4, nt = blockDim.x;
    const float4* src = reinterpret_cast<const float4*>(x);
    const float4* nw4 = reinterpret_cast<const float4*>(norm_w);
    for (int base = 0; base < ng; base += kDpGroupsInFlight * nt) {  // the same trip count in every thread
        float v[kDpGroupsInFlight][8];
#pragma unroll
        for (int u = 0; u < kDpGroupsInFlight; ++u) {
            const int gi = base + u * nt + (int)threadIdx.x;
            const bool live = gi < ng;
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f), o4 = make_float4(1.f, 1.f, 1.f, 1.f);
            const float4 a0 = live ? __ldcg(src + 2 * gi) : z4, a1 = live ? __ldcg(src + 2 * gi + 1) : z4;
            const float4 w0 = live && norm_w ? __ldg(nw4 + 2 * gi) : o4, w1 = live && norm_w ? __ldg(nw4 + 2 * gi + 1) : o4;
            v[u][0] = a0.x * w0.x; v[u][1] = a0.y * w0.y; v[u][2] = a0.z * w0.z; v[u][3] = a0.w * w0.w;
            v[u][4] = a1.x * w1.x; v[u][5] = a1.y * w1.y; v[u][6] = a1.z * w1.z; v[u][7] = a1.w * w1.w;
        }
#pragma unroll
        for (int u = 0; u < kDpGroupsInFlight; ++u) {
            if (base + u * nt >= ng) break;  // uniform over the CTA
            const int gi = base + u * nt + (int)threadIdx.x;
            dp_group_digits<WT>(v[u], gi, gi < ng, xs);
        }
    }
    __syncthreads();
}

// Activation digit records of the integer variant for one sequence (whole CTA):
// rmsnorm by norm_w when given, then per 32-column block the power-of-two
// scale and the balanced base-128 digits, one thread per 8-column group.
// Reads the activations through L2 (the producing kernel wrote them). Ends with
// a CTA barrier.
template <int WT>
__device__ __forceinline__ void dp_build_records(const float* x, const float* norm_w, float eps, int in, uint8_t* xs,
                                                 float* wstat, float* inv) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = in / 32, ng = nb * 4;  // 8-column groups
    const float4* src = reinterpret_cast<const float4*>(x);
    const float4* nw4 = reinterpret_cast<const float4*>(norm_w);
    constexpr int RMAX = 4;  // groups per thread held in registers (rows up to 4 * 8 * blockDim columns)
    const int nt = blockDim.x;
    if (ng > RMAX * nt) {  // too long to hold: the sum of squares first, then the groups round by round
        float ss = 0.f;
        if (norm_w) {
            for (int f = threadIdx.x; f < (in >> 2); f += nt) {
                const float4 v = __ldcg(src + f);
                ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) wstat[warp * 2] = ss;
        __syncthreads();
        float a = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) a += wstat[w * 2];
        const float iv = norm_w ? 1.f / sqrtf(a / float(in) + eps) : 1.f;
        for (int base = 0; base < ng; base += nt) {
            const int gi = base + threadIdx.x;
            const bool live = gi < ng;
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 a0 = live ? __ldcg(src + 2 * gi) : z4, a1 = live ? __ldcg(src + 2 * gi + 1) : z4;
            float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            dp_group_record<WT>(v, norm_w, iv, gi, live, xs);
        }
    } else {  // one load of every group, then the statistics and the records from registers
        float v[RMAX][8];
        float ss = 0.f;
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            const int gi = r * nt + threadIdx.x;
            const bool live = gi < ng;
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 a0 = live ? __ldcg(src + 2 * gi) : z4, a1 = live ? __ldcg(src + 2 * gi + 1) : z4;
            v[r][0] = a0.x; v[r][1] = a0.y; v[r][2] = a0.z; v[r][3] = a0.w;
            v[r][4] = a1.x; v[r][5] = a1.y; v[r][6] = a1.z; v[r][7] = a1.w;
#pragma unroll
            for (int k = 0; k < 8; ++k) ss = fmaf(v[r][k], v[r][k], ss);
        }
        float iv = 1.f;
        if (norm_w) {
            ss = warp_sum(ss);
            if (lane == 0) wstat[warp * 2] = ss;
            __syncthreads();
            float a = 0.f;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) a += wstat[w * 2];
            iv = 1.f / sqrtf(a / float(in) + eps);
        }
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r * nt >= ng) break;  // uniform over the CTA
            const int gi = r * nt + threadIdx.x;
            dp_group_record<WT>(v[r], norm_w, iv, gi, gi < ng, xs);
        }
    }
    (void)nw4;
    if (inv) *inv = 1.f;  // (statistics live in registers; kept for callers that read it)
    __syncthreads();
}

template <int WT, int NT, int EPI, typename KV, int W = kSkWarps>
__global__ void __launch_bounds__(W * 32, 1) mv_sk_kernel(const MvParams p) {
    constexpr int QB = tile_qbytes(WT);
    constexpr int SB = WT == T_F16 ? 0 : kTileSBytes;
    constexpr int KB = sk_kb(WT);
    constexpr int R = sk_stages(WT);
    constexpr int STAGE = sk_stage_bytes(WT);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    constexpr bool DP = NT == 0;  // integer variant, one sequence
    static_assert(!DP || WT != T_F16, "the integer variant takes Q4_0 or Q8_0");
    const int B = DP ? 1 : p.nseq;
    const int nb = p.nb;

    uint8_t* ring = smem + warp * R * STAGE;
    uint8_t* xs = smem + W * R * STAGE;
    float* parts = reinterpret_cast<float*>(xs + (size_t)nb * B * 128);  // [warp][slot][16][B]
    uint8_t* small = reinterpret_cast<uint8_t*>(parts + W * kSkSlots * 16 * B);
    int* tickets = reinterpret_cast<int*>(small);                        // [team leader][slot]
    int* merged = tickets + W * kSkSlots;                         // [team leader][slot] last merged tile + 1
    float* wstat = reinterpret_cast<float*>(merged + W * kSkSlots);  // [warps][B][2]
    float* inv = wstat + W * B * 2;                               // [B] rmsnorm 1/rms
    float* xsc = inv + B;                                                // [B] power-of-two split scale
    uint64_t* bars = reinterpret_cast<uint64_t*>(small + sk_small_bytes(B, W)) + warp * R;

    // this CTA's tiles, this warp's team and K slice (sk_split: the host's arithmetic)
    const int k = p.team_k, teams = p.team_n;
    const SkWarpRange wr = sk_warp_range(p, blockIdx.x, warp);
    const int team = wr.team, leader = wr.leader;
    const int t_lo = wr.t_lo, t_hi = wr.t_hi;
    const int b_lo = wr.b_lo, b_hi = wr.b_hi;  // slice of every tile
    const int slice = b_hi - b_lo;
    const int st_per_tile = (slice + KB - 1) / KB;
    int my_tiles = 0;
    for (int t = t_lo + team; t < t_hi; t += teams) ++my_tiles;
    const int nst = my_tiles * st_per_tile;

    // The warp's stages walk its tiles (t_lo + team + i*teams) and, within each,
    // its slice in KB-block steps. Positions advance incrementally (no divisions).
    int iss_ti = 0, iss_st = 0, iss_slot = 0;  // next stage to issue
    auto issue = [&]() {
        const int t = t_lo + team + iss_ti * teams;
        const int b0 = b_lo + iss_st * KB;
        const int n = min(KB, b_hi - b0);
        const size_t first = (size_t)t * nb + b0;
        uint8_t* dst = ring + iss_slot * STAGE;
        mbar_expect_tx(bars + iss_slot, (uint32_t)(n * (QB + SB)));
        bulk_g2s(dst, p.q + first * QB, (uint32_t)(n * QB), bars + iss_slot);
        if (SB) bulk_g2s(dst + KB * QB, p.s + first * SB, (uint32_t)(n * SB), bars + iss_slot);
        if (++iss_st == st_per_tile) { iss_st = 0; ++iss_ti; }
        if (++iss_slot == R) iss_slot = 0;
    };
    int issued = 0;
    if (lane == 0) {
        for (int r = 0; r < R; ++r) mbar_init(bars + r, 1);
        mbar_fence_init();
        for (; issued < min(R, nst); ++issued) issue();
    }
    for (int i = threadIdx.x; i < 2 * W * kSkSlots; i += blockDim.x) tickets[i] = 0;  // and merged[]
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait();

    // ---- prologue: the whole activation vector -> binary16 hi/lo in fragment order
    //      (integer variant: int8 digit records, one warp per 32-column block)
    if constexpr (DP) {
        if (p.scale_mode != 0) {
            // records of x * norm weight without the 1/rms; the rmsnorm scale comes from the
            // producing kernel's partial sums of squares (mode 1, else unit) and multiplies the
            // finished rows instead. The last warp sums them: with at most (W - 1) * 32 groups
            // (4096 columns at 24 warps) it has no records to build
            if (warp == W - 1) {
                float a = 0.f;
                if (p.scale_mode == 1) {
                    int t = lane;
                    for (; t + 96 < p.ss_tiles; t += 128) {
                        const float v0 = __ldcg(p.ss + t), v1 = __ldcg(p.ss + t + 32);
                        const float v2 = __ldcg(p.ss + t + 64), v3 = __ldcg(p.ss + t + 96);
                        a += (v0 + v1) + (v2 + v3);
                    }
                    for (; t < p.ss_tiles; t += 32) a += __ldcg(p.ss + t);
                    a = warp_sum(a);
                }
                if (lane == 0) xsc[0] = p.scale_mode == 1 ? 1.f / sqrtf(a / float(p.ss_n) + p.eps) : 1.f;
            }
            dp_records_unscaled<WT>(p.x, p.norm_w, nb, xs);
        } else {
            dp_build_records<WT>(p.x, p.norm_w, p.eps, p.in, xs, wstat, inv);
            if (threadIdx.x == 0) xsc[0] = 1.f;  // the digit scales are applied per block
        }
        __syncthreads();
    } else {
        const int nv = p.in >> 2;  // float4 per sequence
#pragma unroll
        for (int s = 0; s < NT * 8; ++s) {
            if (s < B) {
                float ss = 0.f, mx = 0.f;
                const float4* src = reinterpret_cast<const float4*>(p.x + (size_t)s * p.ldx);
                const float4* nw4 = reinterpret_cast<const float4*>(p.norm_w);
#pragma unroll 4
                for (int f = threadIdx.x; f < nv; f += blockDim.x) {
                    const float4 v = src[f];
                    const float4 w = p.norm_w ? nw4[f] : make_float4(1.f, 1.f, 1.f, 1.f);
                    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
                    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * w.x), fabsf(v.y * w.y)), fmaxf(fabsf(v.z * w.z), fabsf(v.w * w.w))));
                }
                ss = warp_sum(ss);
                mx = warp_max(mx);
                if (lane == 0) { wstat[(warp * B + s) * 2] = ss; wstat[(warp * B + s) * 2 + 1] = mx; }
            }
        }
        __syncthreads();
        if (threadIdx.x < B) {
            const int s = threadIdx.x;
            float a = 0.f, m = 0.f;
            for (int w = 0; w < W; ++w) { a += wstat[(w * B + s) * 2]; m = fmaxf(m, wstat[(w * B + s) * 2 + 1]); }
            const float iv = p.norm_w ? 1.f / sqrtf(a / float(p.in) + p.eps) : 1.f;
            m *= iv;
            int ex = 0;
            if (m > 0.f && isfinite(m)) { frexpf(m, &ex); ex = max(-100, min(100, ex)); }
            inv[s] = iv;
            xsc[s] = ldexpf(1.f, ex - 11);  // max |x| * 2^(11-ex) lies in [2^10, 2^11)
        }
        __syncthreads();
        __half* xh = reinterpret_cast<__half*>(xs);
        for (int idx = threadIdx.x; idx < B * nv; idx += blockDim.x) {
            const int s = idx / nv, f = idx % nv;
            const float4 v4 = reinterpret_cast<const float4*>(p.x + (size_t)s * p.ldx)[f];
            const float4 w4 = p.norm_w ? reinterpret_cast<const float4*>(p.norm_w)[f] : make_float4(1.f, 1.f, 1.f, 1.f);
            const float vv[4] = {v4.x, v4.y, v4.z, v4.w}, ww[4] = {w4.x, w4.y, w4.z, w4.w};
            const float up = 1.f / xsc[s];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int e = 4 * f + q;
                float v = vv[q];
                if (p.norm_w) v = v * (inv[s] * ww[q]);
                v *= up;  // exact: a power of two
                const __half hi = __float2half_rn(v);
                const __half lo = __float2half_rn(v - __half2float(hi));
                // column 2s holds the hi part of sequence s, column 2s+1 the lo part
                __half* dst = xh + ((size_t)((e >> 5) * 2 * B + 2 * s) * 4 + ((e >> 3) & 3)) * 8;
                dst[frag_pos(e & 7)] = hi;
                dst[32 + frag_pos(e & 7)] = lo;
            }
        }
        __syncthreads();
    }

    // ---- finish one tile: this warp's partial -> slot; the last of the team adds and runs the epilogue
    float acc[DP ? 1 : NT][4];
    float dacc[2] = {0.f, 0.f};  // integer variant: rows g and g+8 of this lane's columns
    auto finish = [&](int t, int tile_idx) {
        const int slot = tile_idx % kSkSlots;
        float* mine = parts + ((size_t)warp * kSkSlots + slot) * 16 * B;
        if (tile_idx >= kSkSlots) {
            // the slot's previous tile must be merged before this warp overwrites its partial
            if (lane == 0) {
                const long long t0 = clock64();
                while (*reinterpret_cast<volatile int*>(merged + leader * kSkSlots + slot) < tile_idx - kSkSlots + 1) {
                    if (clock64() - t0 > 2000000000LL) { atomicExch(p.err, kErrTeamMerge); break; }
                }
            }
            __syncwarp();
        }
        if constexpr (DP) {
            // the four lanes of a row hold its four 8-column groups
            float r0 = dacc[0], r1 = dacc[1];
            r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
            r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
            r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
            r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
            if (c == 0) { mine[g] = r0; mine[g + 8] = r1; }
            dacc[0] = dacc[1] = 0.f;
        } else {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int sq = j * 4 + c;  // columns 2sq (hi) and 2sq+1 (lo)
                if (sq < B) {
                    mine[g * B + sq] = acc[j][0] + acc[j][1];
                    mine[(g + 8) * B + sq] = acc[j][2] + acc[j][3];
                }
                acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
            }
        }
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(tickets + leader * kSkSlots + slot, 1) == k - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence_block();
        float* fin = mine;  // the team's sum is written over this warp's slot
        for (int e = lane; e < 16 * B; e += 32) {
            float v = 0.f;
            for (int w = 0; w < k; ++w) v += parts[((size_t)(leader + w) * kSkSlots + slot) * 16 * B + e];
            const int s = e % B;
            fin[e] = v * xsc[s];
        }
        if (lane == 0) {
            tickets[leader * kSkSlots + slot] = 0;
            __threadfence_block();
            merged[leader * kSkSlots + slot] = tile_idx + 1;
        }
        __syncwarp();
        const int r0 = t * 16;
        for (int e = lane; e < 16 * B; e += 32) {
            const int rl = e / B, s = e % B, r = r0 + rl;
            if (r >= p.rows) continue;
            const float val = fin[e];
            if (EPI == EPI_STORE) {
                p.out[(size_t)s * p.ldo + r] = val;
            } else if (EPI == EPI_ADD) {
                p.out[(size_t)s * p.ldo + r] += val;
            } else if (EPI == EPI_SWIGLU) {
                if ((rl & 1) == 0) {
                    const float up = fin[(rl + 1) * B + s];
                    p.out[(size_t)s * p.ldo + (r >> 1)] = (val / (1.f + expf(-val))) * up;
                }
            } else {  // EPI_QKV
                const int sl = p.slots[s], ps = p.pos[sl];
                int rr = r, region = 0;
                if (rr >= p.q_rows) { rr -= p.q_rows; region = 1; if (rr >= p.kv_rows) { rr -= p.kv_rows; region = 2; } }
                const int d = rr % p.head_dim;
                float o = val;
                if (region < 2 && d < 2 * p.rope_pairs) {
                    const float2 cs = p.rope_cs[(size_t)ps * p.rope_pairs + (d >> 1)];
                    const float other = fin[(rl ^ 1) * B + s];
                    // adjacent-pair rotation, unfused to keep the reference's rounding
                    if ((d & 1) == 0) o = __fsub_rn(__fmul_rn(val, cs.x), __fmul_rn(other, cs.y));
                    else o = __fadd_rn(__fmul_rn(other, cs.y), __fmul_rn(val, cs.x));
                }
                if (region == 0) {
                    p.out[(size_t)s * p.ldo + rr] = o;
                } else {
                    KV* base = reinterpret_cast<KV*>(region == 1 ? p.kc : p.vc);
                    base[(size_t)sl * p.kv_slot_stride + ((size_t)(rr / p.head_dim) * p.kv_cap + ps) * p.head_dim + d] =
                        kv_from<KV>(o);
                }
            }
        }
        __syncwarp();
        if constexpr (DP && EPI == EPI_ADD) {
            if (p.ss_out) {  // the tile's sum of squares of the new residual (rows r0 + lane), for the next rmsnorm
                const int r = r0 + lane;
                const float xn = lane < 16 && r < p.rows ? p.out[r] : 0.f;
                float sq = xn * xn;
                sq += __shfl_xor_sync(0xffffffffu, sq, 1);
                sq += __shfl_xor_sync(0xffffffffu, sq, 2);
                sq += __shfl_xor_sync(0xffffffffu, sq, 4);
                sq += __shfl_xor_sync(0xffffffffu, sq, 8);
                if (lane == 0) p.ss_out[t] = sq;
            }
        }
    };

    // ---- stream this warp's slices
#pragma unroll
    for (int j = 0; j < (DP ? 1 : NT); ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    // this lane's activation column in each n-tile
    uint32_t xlane[DP ? 1 : NT];  // shared-memory addresses
    const int xstride = DP ? kDpRecBytes : 2 * B * 4 * 16;  // bytes between the records of consecutive blocks
    const DpLane dln = dp_lane(lane);  // (integer variant)
    if constexpr (DP) {
        xlane[0] = smem_u32(xs);  // the block records (tile_block_dp adds this lane's fragment)
    } else {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int col = min(j * 8 + g, 2 * B - 1);
            xlane[j] = smem_u32(xs) + (col * 4 + c) * 16;
        }
    }
    const uint32_t ring_a = smem_u32(ring);
    bool aborted = false;
    int slot = 0, cur_ti = 0, cur_st = 0;
    uint32_t phase = 0;
    for (int s = 0; s < nst; ++s) {
        if (!aborted && !mbar_wait(bars + slot, phase, p.err)) aborted = true;
        const int b0 = b_lo + cur_st * KB;
        const int n = aborted ? 0 : min(KB, b_hi - b0);
        const uint32_t sq = ring_a + slot * STAGE;
        const uint32_t ssc = sq + KB * QB;
        if constexpr (DP) {
            const uint32_t xr = xlane[0] + b0 * kDpRecBytes;
            // two blocks per iteration: a fully unrolled stage made instruction fetch the top stall
            // (measured 2-3 % slower steps on the 8B and 1B shapes)
#pragma unroll 2
            for (int j = 0; j < n; ++j) tile_block_dp<WT>(sq + j * QB, ssc + j * SB, xr + j * kDpRecBytes, dln, lane, dacc);
        } else if (n == KB) {
#pragma unroll
            for (int j = 0; j < KB; ++j) tile_block<WT, NT>(sq + j * QB, ssc + j * SB, xlane, b0 + j, xstride, lane, acc);
        } else {
            for (int j = 0; j < n; ++j) tile_block<WT, NT>(sq + j * QB, ssc + j * SB, xlane, b0 + j, xstride, lane, acc);
        }
        __syncwarp();
        if (lane == 0 && !aborted && s + R < nst) {
            fence_proxy_async_smem();  // this warp's reads of the slot precede the copy that refills it
            issue();
            ++issued;
        }
        if (++slot == R) { slot = 0; phase ^= 1u; }
        if (++cur_st == st_per_tile) {
            finish(t_lo + team + cur_ti * teams, cur_ti);
            cur_st = 0;
            ++cur_ti;
        }
    }
    if (aborted && lane == 0) {
        // leave only after the copies still in flight into this warp's ring have landed
        for (int s = max(0, issued - R); s < issued; ++s) mbar_wait(bars + (s % R), (uint32_t)(s / R) & 1u, p.err);
    }
}

}  // namespace laic
