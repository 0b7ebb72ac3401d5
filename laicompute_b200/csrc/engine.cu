// B200 decode engine behind the C ABI of include/laic_b200.h.
//
// One laic_dev holds a Llama model's weights in HBM (uploaded once per GGUF
// tensor), an FP16 (or FP32) KV cache with `max_seqs` slots, and per-step
// CUDA graphs: a decode step (LlamaRuntime::step + sample, reference
// src/inference_v2.cpp:31-32) is one graph replay whose only host traffic is
// the input ids in and the sampled ids out.
//
// Per layer the step runs four dequant-fused matvec launches and one attention
// launch (reference :31):
//   qkv   rmsnorm(attn_norm) -> fused [Wq;Wk;Wv] -> RoPE -> q, K/V cache append
//   attn  split-K GQA decode attention -> attn
//   o     Wo attn, added into the residual
//   gu    rmsnorm(ffn_norm) -> interleaved [Wgate;Wup] -> silu(g)*u
//   down  Wdown act, added into the residual
// then rmsnorm(output_norm) -> lm_head -> sampler. Kernels use programmatic
// dependent launch so each one's launch and prologue overlap the previous one.
//
// Tensor parallelism (tp_size > 1, one process per GPU): each rank holds
// H/tp query heads and Hkv/tp KV heads (their rows of Wq/Wk/Wv and their KV
// cache), F/tp rows of Wgate/Wup, the matching column slices of Wo and Wdown,
// and V/tp rows of the lm_head. After o and after down the ranks' partial
// products are summed with one in-place NCCL allreduce on the residual (rank
// 0 adds its partial to the residual, the others overwrite it with theirs);
// the lm_head slices are all-gathered so every rank samples the same ids.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <vector>

#include "../../include/laic_b200.h"
#include "allreduce.cuh"
#include "attention.cuh"
#include "launch.cuh"
#include "misc.cuh"
#include "mma_matvec.cuh"
#include "mv_streamk.cuh"
#include "nccl_dl.h"
#include "prefill.cuh"
#include "sampler.cuh"
#include "stream_step.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

#define CK(x)                                                                                      \
    do {                                                                                           \
        cudaError_t e_ = (x);                                                                      \
        if (e_ != cudaSuccess) return fail(LAIC_E_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

using laic::T_F16;
using laic::T_F32;
using laic::T_Q4_0;
using laic::T_Q8_0;
using laic::T_Q5_0;

size_t elem_bytes(int type, size_t n) {
    switch (type) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q4_0: return n / 32 * 18;
    case T_Q8_0: return n / 32 * 34;
    case T_Q5_0: return n / 32 * 22;
    }
    return 0;
}

// Blocks of a type the device holds as another type with identical values (the reference's
// decode, src/quant_v2.cpp:10 and :12), converted on the host before the tile repack:
//  * Q5_0 (d, 32-bit high bits qh, 16 nibble bytes; element o = d * (v - 16) with v the nibble
//    of byte o/2, low for even o, plus bit o of qh as bit 4) -> Q8_0 (the same d, int8 v - 16):
//    d * float(v - 16) is the very product quant_v2::value forms, so the values are identical;
//  * Q4_0 in upstream ggml's nibble order (elements j and j + 16 share byte j, low nibble
//    first) -> the reference's order (element o in byte o/2, low nibble for even o).
// Returns false for a type that needs no conversion.
static bool convert_blocks(int type, const uint8_t* src, size_t nblocks, bool q4_upstream, int* out_type,
                           std::vector<uint8_t>& out) {
    if (type == T_Q5_0) {
        out.resize(nblocks * 34);
        for (size_t b = 0; b < nblocks; ++b) {
            const uint8_t* p = src + b * 22;
            uint8_t* o = out.data() + b * 34;
            uint32_t qh;
            std::memcpy(&qh, p + 2, 4);
            o[0] = p[0];
            o[1] = p[1];
            for (int e = 0; e < 32; ++e) {
                const uint8_t z = p[6 + e / 2];
                const int v = ((e & 1) ? z >> 4 : z & 15) | (int)(((qh >> e) & 1u) << 4);
                o[2 + e] = (uint8_t)(int8_t)(v - 16);
            }
        }
        *out_type = T_Q8_0;
        return true;
    }
    if (type == T_Q4_0 && q4_upstream) {
        out.resize(nblocks * 18);
        for (size_t b = 0; b < nblocks; ++b) {
            const uint8_t* p = src + b * 18;
            uint8_t* o = out.data() + b * 18;
            o[0] = p[0];
            o[1] = p[1];
            for (int k = 0; k < 16; ++k) {  // byte k holds elements 2k and 2k+1 in the reference's order
                auto nib = [&](int e) { return e < 16 ? p[2 + e] & 15 : p[2 + e - 16] >> 4; };
                o[2 + k] = (uint8_t)(nib(2 * k) | (nib(2 * k + 1) << 4));
            }
        }
        *out_type = T_Q4_0;
        return true;
    }
    return false;
}

// A projection matrix in the fragment-tile layout of mma_matvec.cuh.
struct Mat {
    int type = -1;
    int rows = 0, ntiles = 0, in = 0, nb = 0;
    uint8_t* q = nullptr;
    uint8_t* s = nullptr;
    size_t bytes() const {  // GGUF bytes of the matrix: what one matvec must stream
        return elem_bytes(type, (size_t)rows * in);
    }
};

int mat_alloc(Mat& m, int type, int rows, int in) {
    if (type != T_F16 && type != T_Q4_0 && type != T_Q8_0)
        return fail(LAIC_E_UNSUPPORTED, "unsupported matrix type " + std::to_string(type) + " (F16, Q8_0, Q4_0 only)");
    if (in % 32) return fail(LAIC_E_UNSUPPORTED, "row length must be a multiple of 32");
    m.type = type; m.rows = rows; m.in = in; m.nb = in / 32; m.ntiles = (rows + 15) / 16;
    const size_t qbytes = (size_t)m.ntiles * m.nb * laic::tile_qbytes(type);
    CK(cudaMalloc(&m.q, qbytes));
    CK(cudaMemset(m.q, 0, qbytes));
    if (type != T_F16) {
        const size_t sbytes = (size_t)m.ntiles * m.nb * laic::kTileSBytes;
        CK(cudaMalloc(&m.s, sbytes));
        CK(cudaMemset(m.s, 0, sbytes));
    }
    return LAIC_OK;
}

void mat_free(Mat& m) {
    if (m.q) cudaFree(m.q);
    if (m.s) cudaFree(m.s);
    m.q = nullptr; m.s = nullptr;
}

// Copy GGUF rows (raw block bytes) into matrix rows r*row_mul + row_add
// through a device staging buffer, repacking into fragment tiles.
int mat_fill(Mat& m, const uint8_t* host, int nrows, int row_mul, long long row_add, cudaStream_t st) {
    const size_t row_bytes = elem_bytes(m.type, (size_t)m.in);
    const size_t chunk_rows = std::max<size_t>(1, (64u << 20) / row_bytes);
    void* staging = nullptr;
    CK(cudaMalloc(&staging, std::min<size_t>(chunk_rows, (size_t)nrows) * row_bytes));
    for (size_t r0 = 0; r0 < (size_t)nrows; r0 += chunk_rows) {
        const size_t n = std::min(chunk_rows, (size_t)nrows - r0);
        CK(cudaMemcpyAsync(staging, host + r0 * row_bytes, n * row_bytes, cudaMemcpyHostToDevice, st));
        laic::repack_tiles_kernel<<<1184, 256, 0, st>>>(m.type, (const uint8_t*)staging, (long long)n, m.nb, row_mul,
                                                        (long long)r0 * row_mul + row_add, m.q, m.s);
        CK(cudaGetLastError());
        CK(cudaStreamSynchronize(st));
    }
    cudaFree(staging);
    return LAIC_OK;
}

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------
using laic::launch_k;

int g_num_sms = 0;
int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

// Launch shape of one fragment-tile matvec: n-tiles, K split, ring, grid, shared memory.
struct MvShape {
    bool sk = false;  // team kernel (small batches whose activations fit in shared memory)
    int warps = laic::kSkWarps;  // team kernel: warps per CTA
    int nt = 1, nk = 1, kr = 1, kb = 1, stages = 2, grid = 1;
    int groups = 1, sgrp = 1;  // tile kernel: sequence groups (grid.y) of sgrp sequences
    bool wide = false;         // the wide kernel (EPI_STORE, warps own whole row tiles)
    size_t smem = 0;
    size_t part_floats = 0;  // split-K scratch it needs
};

constexpr size_t kSmemBudget = 220 * 1024;

// Largest batch the team kernel takes; larger batches go to the tile kernel.
#ifndef LAIC_SK_MAX_BATCH
#define LAIC_SK_MAX_BATCH 16
#endif
// Models with at most this many projection weights per layer run every batch from
// LAIC_TILE_MIN_BATCH up on the tile kernel with activation records.
#ifndef LAIC_SMALL_LAYER_WEIGHTS
#define LAIC_SMALL_LAYER_WEIGHTS 16.0e6
#endif
#ifndef LAIC_TILE_MIN_BATCH
#define LAIC_TILE_MIN_BATCH 1
#endif
// One-sequence steps of larger models pass the team kernel's integer records between
// the projections (0: every projection builds them from x itself).
#ifndef LAIC_DP_RECORDS
#define LAIC_DP_RECORDS 1
#endif
// In such steps the lm_head stays on the team kernel up to this batch.
#ifndef LAIC_LM_TEAM_MAX_BATCH
#define LAIC_LM_TEAM_MAX_BATCH 4
#endif

// team_ok false: the tile kernel whatever the batch (a step whose projections pass activation
// records between them).
// store: an EPI_STORE launch, which may take the wide kernel.
MvShape mv_shape(const Mat& m, int B, bool team_ok = true, bool store = false) {
    MvShape sh;
    if (team_ok && B <= LAIC_SK_MAX_BATCH) {
        // one sequence of Q4_0 / Q8_0: integer dot products (nt 0); else hi and lo columns side by side
        const int nt = (B == 1 && m.type != T_F16) ? 0 : B <= 4 ? 1 : B <= 8 ? 2 : 4;
        int warps = laic::sk_warps_for(m.type, nt, m.nb, m.rows);
        size_t smem = laic::sk_smem_bytes(m.type, m.nb, B, warps);
        if (smem > kSmemBudget && warps != laic::kSkWarps) {
            warps = laic::kSkWarps;
            smem = laic::sk_smem_bytes(m.type, m.nb, B, warps);
        }
        if (smem <= kSmemBudget) {
            sh.sk = true;
            sh.warps = warps;
            sh.nt = nt;
            sh.grid = std::max(1, std::min(num_sms(), m.ntiles));  // each CTA owns whole row tiles
            sh.smem = smem;
            sh.part_floats = 0;
            return sh;
        }
    }
    const int G = num_sms();
    const int b8 = (B + 7) / 8 * 8;
    if (store) {
        // many row tiles: the wide kernel, with two ring stages per warp where they fit, then one;
        // the largest sequence group that fits (each group streams the matrix once more from L2)
        for (int S : {16, 8})
            for (int sgrp : {b8, 32, 16, 8}) {
                if (sgrp != b8 && sgrp >= b8) continue;
                const size_t smem = laic::mv_wide_smem(m.type, m.nb, sgrp, S);
                if (smem > kSmemBudget) continue;
                const int groups = (B + sgrp - 1) / sgrp;
                const int cta = G / groups;
                if (cta < 1 || m.ntiles < 16 * cta) continue;  // at least two tiles per warp
                sh.wide = true;
                sh.nt = sgrp <= 8 ? 1 : sgrp <= 16 ? 2 : sgrp <= 32 ? 4 : 8;
                sh.sgrp = sgrp;
                sh.groups = groups;
                sh.grid = cta;
                sh.stages = S;
                sh.nk = 1;
                sh.kr = m.nb;
                sh.smem = smem;
                return sh;
            }
    }
    sh.kb = m.type == T_F16 ? 16 : 32;
    const size_t sbytes = m.type == T_F16 ? 0 : laic::kTileSBytes;
    const size_t stage_bytes = (size_t)sh.kb * (laic::tile_qbytes(m.type) + sbytes);
    // rough microseconds: a consumer warp's tile-block (mma count grows with the n-tiles), a tile's
    // reduction and epilogue, the CTA's activation copy (~150 KB/us per SM from L2), and the
    // split-K merge (partials to L2, fence, ticket, second pass)
    const double t_tile = 1.0, t_merge = 4.0, x_kb_per_us = 150.0;
    double best = 1e30;
    for (int sgrp : {b8, 32, 16, 8}) {  // sequences per group (whole n-tiles); groups = grid.y
        if (sgrp != b8 && sgrp >= b8) continue;  // smaller groups only
        const int groups = (B + sgrp - 1) / sgrp;
        const int nt = sgrp <= 8 ? 1 : sgrp <= 16 ? 2 : sgrp <= 32 ? 4 : 8;
        const double t_blk = 0.05 + 0.025 * nt;
        const size_t fixed = (size_t)laic::kConsumerWarps * 16 * nt * 8 * 4 + 16 * (size_t)sgrp * 4 + nt * 8 * 8 + 1024;
        for (int nk = 1; nk <= std::min(m.nb, 64); ++nk) {
            const int kr = (m.nb + nk - 1) / nk;
            if ((m.nb + kr - 1) / kr != nk) continue;  // no empty split
            const size_t xs = (size_t)kr * sgrp * 128;
            if (fixed + xs + 2 * stage_bytes > kSmemBudget) continue;
            const int cta_per_k = G / (nk * groups);
            if (cta_per_k < 1) break;
            const int tiles_per = (m.ntiles + cta_per_k - 1) / cta_per_k;
            const int blk_rounds = (kr + laic::kConsumerWarps - 1) / laic::kConsumerWarps;
            const double cost = (double)tiles_per * (blk_rounds * t_blk + t_tile) + xs / 1024.0 / x_kb_per_us +
                                (nk > 1 ? t_merge : 0.0);
            if (cost < best - 1e-9) {
                best = cost;
                sh.nt = nt;
                sh.groups = groups;
                sh.sgrp = sgrp;
                sh.nk = nk;
                sh.kr = kr;
                sh.stages = (int)std::min<size_t>(8, (kSmemBudget - fixed - xs) / stage_bytes);
                sh.grid = nk * std::min(cta_per_k, m.ntiles);
                sh.smem = fixed + xs + sh.stages * stage_bytes;
            }
        }
    }
    sh.part_floats = sh.nk > 1 ? (size_t)m.ntiles * sh.nk * 16 * B : 0;
    return sh;
}

// Scratch shared by every matvec launch of a stream (launches are serialised):
// split-K partials and tickets, and the prepared activations of the tile kernel.
struct MvScratch {
    float* part = nullptr;
    unsigned* tile_cnt = nullptr;
    int* err = nullptr;
    uint8_t* xg = nullptr;
    float* xinv = nullptr;
    size_t part_cap = 0, cnt_cap = 0, xg_cap = 0, xinv_cap = 0;
};

struct MvNeed {  // scratch one launch shape needs
    size_t part_floats = 0, ntiles = 0, xg_bytes = 0, xinv_floats = 0;
    void merge(const MvNeed& o) {
        part_floats = std::max(part_floats, o.part_floats);
        ntiles = std::max(ntiles, o.ntiles);
        xg_bytes = std::max(xg_bytes, o.xg_bytes);
        xinv_floats = std::max(xinv_floats, o.xinv_floats);
    }
};

MvNeed mv_need(const Mat& m, int B) {
    MvNeed n;
    for (int v = 0; v < 4; ++v) {  // team or tile, store or not: whichever kernel may run this shape
        const MvShape sh = mv_shape(m, B, v & 1, v & 2);
        MvNeed k;
        k.part_floats = sh.part_floats;
        k.ntiles = (size_t)m.ntiles * sh.groups;  // tickets per (row tile, group)
        if (!sh.sk) {
            k.xg_bytes = (size_t)m.nb * B * 128;
            k.xinv_floats = (size_t)sh.nk * B;
        }
        n.merge(k);
    }
    return n;
}

// Grow the scratch to `need`; returns whether any buffer moved (captured graphs are stale then).
int mv_scratch_reserve(MvScratch& sc, const MvNeed& need, bool* moved = nullptr) {
    bool mv = false;
    if (!sc.err) {
        CK(cudaMalloc(&sc.err, 4));
        CK(cudaMemset(sc.err, 0, 4));
    }
    if (need.part_floats > sc.part_cap) {
        if (sc.part) cudaFree(sc.part);
        sc.part = nullptr;
        CK(cudaMalloc(&sc.part, need.part_floats * 4));
        sc.part_cap = need.part_floats;
        mv = true;
    }
    if (need.ntiles > sc.cnt_cap) {
        if (sc.tile_cnt) cudaFree(sc.tile_cnt);
        sc.tile_cnt = nullptr;
        CK(cudaMalloc(&sc.tile_cnt, need.ntiles * 4));
        CK(cudaMemset(sc.tile_cnt, 0, need.ntiles * 4));
        sc.cnt_cap = need.ntiles;
        mv = true;
    }
    if (need.xg_bytes > sc.xg_cap) {
        if (sc.xg) cudaFree(sc.xg);
        sc.xg = nullptr;
        CK(cudaMalloc(&sc.xg, need.xg_bytes));
        sc.xg_cap = need.xg_bytes;
        mv = true;
    }
    if (need.xinv_floats > sc.xinv_cap) {
        if (sc.xinv) cudaFree(sc.xinv);
        sc.xinv = nullptr;
        CK(cudaMalloc(&sc.xinv, need.xinv_floats * 4));
        sc.xinv_cap = need.xinv_floats;
        mv = true;
    }
    if (moved) *moved = mv;
    return LAIC_OK;
}

void mv_scratch_free(MvScratch& sc) {
    if (sc.part) cudaFree(sc.part);
    if (sc.tile_cnt) cudaFree(sc.tile_cnt);
    if (sc.err) cudaFree(sc.err);
    if (sc.xg) cudaFree(sc.xg);
    if (sc.xinv) cudaFree(sc.xinv);
    sc = MvScratch{};
}

// What a producing kernel left for a projection: the tile kernel's activation records (xg), and
// the rmsnorm's partial sums of squares (mode 1) or a unit scale (mode 2).
struct RecIn {
    const uint8_t* xg = nullptr;
    int mode = 0;             // 1: rmsnorm scale from ss; 2: unit scale
    const float* ss = nullptr;
    int ss_tiles = 0;
    bool dp = false;          // one sequence on the team kernel's integer variant: it builds its records
                              // from x and takes only mode / ss from here
};

// One projection: the team kernel for small batches, else activation
// preparation (unless `rin` brings the records) + tile kernel. `launches`
// counts the kernels enqueued.
cudaError_t launch_matvec(const Mat& m, laic::MvParams p, int epi, bool kv32, const MvScratch& sc, cudaStream_t st,
                          bool pdl, int* launches = nullptr, const RecIn* rin = nullptr, bool team_ok = true) {
    const MvShape sh = mv_shape(m, p.nseq, team_ok, epi == laic::EPI_STORE);
    p.q = m.q; p.s = m.s; p.rows = m.rows; p.ntiles = m.ntiles; p.in = m.in; p.nb = m.nb;
    if (sh.sk) {
        p.err = sc.err;
        if (rin && rin->dp && sh.nt == 0) {  // records from x, the rmsnorm scale from the partial sums
            p.scale_mode = rin->mode; p.ss = rin->ss; p.ss_tiles = rin->ss_tiles; p.ss_n = m.in;
        }
        laic::sk_split(p, sh.grid, sh.warps);
        if (launches) *launches += 1;
        return laic::mv_sk_launch(m.type, sh.nt, epi, kv32, p, sh.grid, sh.smem, st, pdl, sh.warps);
    }
    p.nk = sh.nk; p.kr = sh.kr; p.kb = sh.kb; p.stages = sh.stages; p.sgrp = sh.sgrp;
    p.part = sc.part; p.tile_cnt = sc.tile_cnt; p.err = sc.err;
    if (rin && rin->xg && !rin->dp) {
        p.xg = rin->xg; p.scale_mode = rin->mode; p.ss = rin->ss; p.ss_tiles = rin->ss_tiles; p.ss_n = m.in;
    } else {
        laic::XPrepParams xp{p.x, p.ldx, p.norm_w, p.eps, m.in, m.nb, p.nseq, sh.kr, sc.xg, sc.xinv};
        cudaError_t e = laic::xprep_launch(xp, sh.nk, st, pdl);
        if (e != cudaSuccess) return e;
        p.xg = sc.xg; p.xinvg = sc.xinv; p.scale_mode = 0;
        if (launches) *launches += 1;
    }
    if (launches) *launches += 1;
    if (sh.wide) return laic::mv_wide_launch(m.type, sh.nt, p, sh.grid, sh.groups, sh.smem, st, pdl);
    return laic::mv_launch(m.type, sh.nt, epi, kv32, p, sh.grid, sh.groups, sh.smem, st, pdl);
}

using AttnFn = void (*)(laic::AttnParams);
template <int D, int GM>
AttnFn attn_fn_g(bool kv32, bool cl) {
    if (kv32) return laic::attn_decode_kernel<D, GM, float, true>;
    return cl ? laic::attn_mma_kernel<D, GM, true> : laic::attn_mma_kernel<D, GM, false>;
}
template <int D>
AttnFn attn_fn_d(int G, bool kv32, bool cl) {
    if (G <= 1) return attn_fn_g<D, 1>(kv32, cl);
    if (G <= 2) return attn_fn_g<D, 2>(kv32, cl);
    if (G <= 4) return attn_fn_g<D, 4>(kv32, cl);
    return attn_fn_g<D, 8>(kv32, cl);
}
// FP32 KV (parity mode): the register kernel with the reference's score order;
// FP16 KV: the tensor-core kernel over chunks staged in shared memory, its splits merged
// inside a thread-block cluster (cl) or through global scratch.
AttnFn attn_pick(int D, int G, bool kv32, bool cl = false) {
    if (D == 32) return attn_fn_d<32>(G, kv32, cl);
    if (D == 64) return attn_fn_d<64>(G, kv32, cl);
    if (D == 128) return attn_fn_d<128>(G, kv32, cl);
    return nullptr;
}
// Cluster merge for 2..8 splits of the tensor-core kernel.
bool attn_cluster(int nsplit, bool kv32) { return !kv32 && nsplit >= 2 && nsplit <= laic::kAttnMaxCluster; }
size_t attn_smem(int D, bool kv32, int nbuf = 1) { return kv32 ? 0 : (size_t)nbuf * laic::attn_chunk_smem(D); }
// Chunk buffers of the tensor-core attention: with enough (sequence, kv head) pairs to fill
// the GPU, a split takes up to this many chunks, all fetched before the dependency wait,
// so short contexts need no split merge.
int attn_max_nbuf(int D) { return D <= 64 ? 3 : 2; }

// ---------------------------------------------------------------------------
// the engine
// ---------------------------------------------------------------------------
struct Layer {
    Mat qkv, o, gu, down;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    unsigned have = 0;  // bit per uploaded tensor
};
enum : unsigned { H_ANORM = 1, H_Q = 2, H_K = 4, H_V = 8, H_O = 16, H_FNORM = 32, H_GATE = 64, H_UP = 128, H_DOWN = 256,
                  H_ALL = 511 };

// MODE_SPEC0 / MODE_SPEC1: a speculative step of laic_dev_step, inputs like MODE_CHAIN (the
// previous step's sampled ids, slots and parameters already on the device), outputs like
// MODE_STEP (ids and error words copied to pinned host memory: buffer 0 or 1, so that the
// next guess can be queued before this one's outputs are read).
enum StepMode : int { MODE_PREFILL = 0, MODE_STEP = 1, MODE_CHAIN = 2, MODE_SPEC0 = 3, MODE_SPEC1 = 4 };

}  // namespace

struct laic_dev {
    laic_dev_desc a{};
    laic_dev_opts o{};
    int device = 0;
    cudaStream_t st = nullptr;
    // H, Hkv, kv (= Hkv * D), hq (= H * D) and F are this rank's shares; h and V are the full sizes
    int H = 0, Hkv = 0, D = 0, G = 0, h = 0, kv = 0, hq = 0, F = 0, V = 0, Vl = 0, L = 0, S = 0, cap = 0,
        rope_pairs = 0;
    bool kv32 = false, use_graph = true, use_pdl = true;
    int tp = 1, tr = 0;  // tensor-parallel size and rank
    laic::ncclComm_t comm = nullptr;
    const laic::NcclApi* nccl = nullptr;
    // one-shot peer-memory allreduce of the residual (else NCCL): mailboxes of every rank
    bool ar_p2p = false;
    laic::ArParams ar{};
    float* ar_box = nullptr;      // this rank's mailbox data
    unsigned* ar_flags = nullptr; // this rank's mailbox flags
    unsigned* ar_ctr = nullptr;   // [epoch, done]
    float *logits_l = nullptr, *logits_g = nullptr;  // tp > 1: this rank's vocabulary rows; every rank's
    bool have_lm = false;  // tp > 1: lm holds this rank's lm_head rows

    // one sequence: the persistent decode-step kernel (stream_step.cuh) and its state
    laic::LsLayer* ls_layers = nullptr;
    uint8_t *ls_rec_x = nullptr, *ls_rec_attn = nullptr, *ls_rec_act = nullptr;
    float *ls_ss = nullptr, *ls_apart = nullptr;
    unsigned* ls_head_tick = nullptr;
    unsigned long long *ls_done = nullptr, *ls_epoch = nullptr;
    size_t ls_done_bytes = 0;
    int ls_type = -1, ls_nst = 0, ls_maxch = 0, ls_runs = 0;
    size_t ls_smem_bytes = 0;
    bool ls_ready = false, ls_checked = false, use_ls = true, force_ls = false, ls_lm = false;
    bool q4_upstream = false;  // Q4_0 uploads arrive in upstream ggml's nibble order
    // Speculative next step of laic_dev_step: after a step whose tokens were the previous step's
    // sampled ids (same slots and parameters), one more step runs on the device's own ids while
    // the host takes its answer; the next call uses it when it brings exactly those tokens again,
    // else undoes it (positions, repeat-penalty counts, error words) before its own step.
    bool use_spec = true;
    bool spec_pending = false;
    int last_nseq = 0;
    std::vector<int32_t> last_slots;
    std::vector<uint32_t> last_ids;      // ids the last step returned: the speculative step's tokens
    std::vector<laic::SampleDev> last_params;
    int spec_buf = 0;                    // host output buffer of the pending guess
    cudaEvent_t spec_ev[2] = {nullptr, nullptr};  // recorded after the guess writing buffer 0 / 1
    int* d_spec = nullptr;               // [2][max_seqs]: tokens and positions to restore on a rollback
    int* h_spec = nullptr;               // pinned staging of the same

    // Wait for a pending speculative step and undo it (the caller is about to change the state it
    // assumed). No-op without one.
    int spec_cancel() {
        if (!spec_pending) return LAIC_OK;
        spec_pending = false;
        CK(cudaStreamSynchronize(st));
        const int n = last_nseq;
        for (int i = 0; i < n; ++i) {
            h_spec[i] = (int)last_ids[i];
            h_spec[S + i] = (int)h_pos[last_slots[i]];
        }
        CK(cudaMemcpyAsync(d_spec, h_spec, 2 * S * sizeof(int), cudaMemcpyHostToDevice, st));
        CK(cudaMemcpyAsync(d_slots, last_slots.data(), n * sizeof(int), cudaMemcpyHostToDevice, st));
        laic::unstep_kernel<<<1, 256, 0, st>>>(d_slots, (const unsigned*)d_spec, d_spec + S, pos, counts, V, n);
        CK(cudaGetLastError());
        CK(cudaMemsetAsync(mvs.err, 0, 4, st));  // the discarded step's wait or sampler errors are not the caller's
        CK(cudaMemsetAsync(d_err, 0, 4, st));
        CK(cudaStreamSynchronize(st));
        const bool waits_failed = h_err[2 * spec_buf] != 0;
        h_err[0] = h_err[1] = h_err[2] = h_err[3] = 0;
        if (waits_failed)
            if (int rc = ls_reset()) return rc;  // a failed wait may have left the step kernel's counters part-way
        return LAIC_OK;
    }
    unsigned long long* ls_trace = nullptr;  // LAIC_FLAG_TRACE: per-phase stamps of the last step kernel
    bool trace_on = false;
    // more than 16 sequences on one GPU: binary16 hi/lo activation records written by the producing
    // kernels (embedding, o/down residual epilogues, SwiGLU) for the tile-kernel projections
    uint8_t *rec_x = nullptr, *rec_act = nullptr, *rec_attn = nullptr;

    // batched prompt prefill (tensor-core GEMMs over the prompt's tokens)
    static constexpr int kPfRows = 512;  // tokens per pass
    float *pf_x = nullptr, *pf_c = nullptr, *pf_q = nullptr, *pf_attn = nullptr;
    __half *pf_a = nullptr, *pf_w = nullptr;
    int *pf_slots = nullptr, *pf_npos = nullptr;
    unsigned* pf_tokens = nullptr;
    void* pf_ws = nullptr;
    size_t pf_ws_bytes = 0;
    float* rec_ss = nullptr;  // [h / 16 row tiles][max_seqs] sums of squares of the residual

    Mat embd, lm;
    bool have_embd = false, have_out = false, have_onorm = false;
    float* out_norm = nullptr;
    std::vector<Layer> layers;

    float *x = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr;
    void *kc = nullptr, *vc = nullptr;
    long long kv_layer_stride = 0, kv_slot_stride = 0;
    int* pos = nullptr;
    unsigned* counts = nullptr;
    float2* rope_cs = nullptr;
    float* attn_part = nullptr;
    unsigned* attn_cnt = nullptr;
    int max_split = 1;

    unsigned *d_tokens = nullptr, *d_out_ids = nullptr, *d_hist = nullptr;
    int *d_slots = nullptr, *d_err = nullptr, *d_hist_count = nullptr;
    size_t hist_cap = 0;  // entries of d_hist
    laic::SampleDev* d_params = nullptr;
    unsigned *h_tokens = nullptr, *h_out_ids = nullptr;
    int* h_err = nullptr;  // pinned [2][2]: a step's copies of the two device error flags (matvec waits, sampler)
    float* samp_v = nullptr;  // sampler slices: [S][kSampleSlices] maxima, ids and per-sequence tickets
    int* samp_i = nullptr;
    unsigned* samp_cnt = nullptr;
    int* h_slots = nullptr;
    laic::SampleDev* h_params = nullptr;
    std::vector<long long> h_pos;

    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;  // (nseq, mode) -> graph
    MvScratch mvs;  // split-K partials and tickets of the matvec launches
    int last_split = 1;

    // ------------------------------------------------------------------
    // Steps whose projections all run on the tile kernel, passing activation records from
    // each producing epilogue to the next projection: batches past the team kernel's, and
    // any batch of a model with small layers (there every launch is latency-bound and the
    // records save the norm and activation preparation of each projection).
    bool small_layers() const {
        const double per_layer = (double)h * (hq + 2.0 * kv) + (double)hq * h + 3.0 * h * F;
        return per_layer <= LAIC_SMALL_LAYER_WEIGHTS;
    }
    bool tile_step(int nseq) const {
        return tp == 1 && (nseq > LAIC_SK_MAX_BATCH || (small_layers() && nseq >= LAIC_TILE_MIN_BATCH));
    }

    int attn_nbuf(int nseq) const { (void)nseq; return kv32 ? 1 : attn_max_nbuf(D); }

    int nsplit_for(int nseq) const {
        const int pairs = nseq * Hkv;
        if (kv32) {
            const int s = (8 * num_sms() + pairs - 1) / pairs;  // about eight CTAs per SM
            return std::max(1, std::min(s, max_split));
        }
        // chunked kernel: at most one split per chunk of the capacity, about four CTAs per SM,
        // no more CTAs than stay resident at once, and at most one cluster of splits per pair
        const int chunks = (cap + laic::kAttnChunk - 1) / laic::kAttnChunk;
        int s = (4 * num_sms() + pairs - 1) / pairs;
        const int per_sm = (int)((227 * 1024) / attn_smem(D, false, attn_nbuf(nseq)));
        s = std::min(s, num_sms() * per_sm / pairs);
        s = std::min(s, laic::kAttnMaxCluster);
        return std::max(1, std::min(std::min(s, chunks), max_split));
    }

    bool ready(std::string& missing) const {
        if (!have_embd) { missing = "token_embd.weight"; return false; }
        if (tp == 1 && !have_out && embd.rows != V) { missing = "output.weight"; return false; }
        if (tp > 1 && !have_lm) { missing = "output.weight"; return false; }
        if (!have_onorm) { missing = "output_norm.weight"; return false; }
        for (int l = 0; l < L; ++l) {
            if ((layers[l].have & H_ALL) != H_ALL) {
                static const char* nm[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                           "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
                for (int b = 0; b < 9; ++b)
                    if (!(layers[l].have & (1u << b))) { missing = "blk." + std::to_string(l) + "." + nm[b] + ".weight"; break; }
                return false;
            }
        }
        return true;
    }

    const Mat& lm_head() const { return (have_out || tp > 1) ? lm : embd; }
    int launches_step = 0, launches_prefill = 0;  // kernels in the last enqueued step / prefill

    // Enqueue one step. `timer` (nullable) records events around launches for profiling.
    struct Timer {
        std::vector<std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>> ev;
        std::vector<double> bytes;
    };

    // Tensor parallel: sum the ranks' partial o / down products held in the residual.
    template <typename TB, typename TE>
    int allreduce_residual(int nseq, cudaStream_t s, TB& t_begin, TE& t_end, int* nl) {
        if (tp == 1) return LAIC_OK;
        t_begin("allreduce", 8.0 * nseq * h * (tp - 1) / tp);
        if (ar_p2p) {
            laic::ArParams ap = ar;
            ap.x = x; ap.n = nseq * h;
            CK(launch_k(laic::allreduce_oneshot_kernel, dim3(laic::kArCtas), dim3(laic::kArThreads), 0, s, use_pdl, ap));
            ++*nl;
        } else {
            const laic::ncclResult_t r = nccl->AllReduce(x, x, (size_t)nseq * h, laic::ncclFloat32, laic::ncclSum, comm, s);
            if (r != laic::ncclSuccess) return fail(LAIC_E_NCCL, std::string("ncclAllReduce: ") + nccl->GetErrorString(r));
        }
        t_end();
        return LAIC_OK;
    }

    // Map every rank's mailbox (CUDA IPC handles exchanged with one NCCL all-gather). Leaves
    // ar_p2p false, and NCCL in charge, if a rank cannot map a peer.
    int setup_p2p_allreduce() {
        if (tp < 2 || tp > laic::kArMaxRanks) return LAIC_OK;
        const int nmax = S * h;
        CK(cudaMalloc(&ar_box, (size_t)2 * tp * nmax * 4));
        CK(cudaMalloc(&ar_flags, (size_t)2 * tp * laic::kArCtas * 4));
        CK(cudaMemset(ar_flags, 0, (size_t)2 * tp * laic::kArCtas * 4));
        CK(cudaMalloc(&ar_ctr, 8));
        CK(cudaMemset(ar_ctr, 0, 8));
        cudaIpcMemHandle_t hd[2];
        CK(cudaIpcGetMemHandle(&hd[0], ar_box));
        CK(cudaIpcGetMemHandle(&hd[1], ar_flags));
        const size_t hb = sizeof hd;
        void* dev = nullptr;
        CK(cudaMalloc(&dev, hb * (tp + 1)));
        CK(cudaMemcpy((char*)dev + hb * tp, hd, hb, cudaMemcpyHostToDevice));
        const laic::ncclResult_t r = nccl->AllGather((char*)dev + hb * tp, dev, hb / 4, laic::ncclFloat32, comm, st);
        if (r != laic::ncclSuccess) { cudaFree(dev); return fail(LAIC_E_NCCL, std::string("ncclAllGather: ") + nccl->GetErrorString(r)); }
        std::vector<cudaIpcMemHandle_t> all(2 * tp);
        CK(cudaStreamSynchronize(st));
        CK(cudaMemcpy(all.data(), dev, hb * tp, cudaMemcpyDeviceToHost));
        cudaFree(dev);
        ar = laic::ArParams{};
        ar.rank = tr; ar.ranks = tp; ar.nmax = nmax; ar.epoch = ar_ctr; ar.done = ar_ctr + 1;
        bool ok = true;
        for (int q = 0; q < tp && ok; ++q) {
            if (q == tr) { ar.box[q] = ar_box; ar.flags[q] = ar_flags; continue; }
            void *pb = nullptr, *pf = nullptr;
            if (cudaIpcOpenMemHandle(&pb, all[2 * q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
                cudaIpcOpenMemHandle(&pf, all[2 * q + 1], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = false;
                break;
            }
            ar.box[q] = (float*)pb; ar.flags[q] = (unsigned*)pf;
        }
        ar_p2p = ok;
        return LAIC_OK;
    }

    int enqueue(int nseq, int mode, cudaStream_t s, Timer* timer) {
        const bool full = mode != MODE_PREFILL;
        const bool pdl = use_pdl && !timer;
        // o and down: rank 0 adds its partial to the residual, the other ranks store theirs (then allreduce)
        const int residual_epi = (tp > 1 && tr != 0) ? laic::EPI_STORE : laic::EPI_ADD;
        int nl = 0;  // kernels enqueued
        auto t_begin = [&](const char* name, double b) {
            if (!timer) return;
            cudaEvent_t e0, e1;
            cudaEventCreate(&e0);
            cudaEventCreate(&e1);
            cudaEventRecord(e0, s);
            timer->ev.push_back({name, {e0, e1}});
            timer->bytes.push_back(b);
        };
        auto t_end = [&]() {
            if (timer) cudaEventRecord(timer->ev.back().second.second, s);
        };
        if (mode == MODE_PREFILL || mode == MODE_STEP) {  // chained / speculative steps read the ids the previous step sampled
            CK(cudaMemcpyAsync(d_tokens, h_tokens, nseq * sizeof(unsigned), cudaMemcpyHostToDevice, s));
            CK(cudaMemcpyAsync(d_slots, h_slots, nseq * sizeof(int), cudaMemcpyHostToDevice, s));
            if (full) CK(cudaMemcpyAsync(d_params, h_params, nseq * sizeof(laic::SampleDev), cudaMemcpyHostToDevice, s));
        }

        const bool step_path = nseq == 1 && ls_ready;
        const bool recs = !step_path && tile_step(nseq) && rec_x;  // records travel between the tile-kernel projections
        // one sequence on the team kernel's integer variant: each projection builds its digit
        // records from x; the producers of an rmsnorm input (embedding, o, down) write the
        // partial sums of squares its 1/rms comes from
        auto dp_mat = [](const Mat& m) {
            if (m.type != T_Q4_0 && m.type != T_Q8_0) return false;
            const MvShape sh = mv_shape(m, 1);
            return sh.sk && sh.nt == 0;
        };
        bool dprecs = LAIC_DP_RECORDS && !step_path && !recs && nseq == 1 && tp == 1 && !kv32 && rec_x != nullptr;
        for (int l = 0; l < L && dprecs; ++l)
            dprecs = dp_mat(layers[l].qkv) && dp_mat(layers[l].o) && dp_mat(layers[l].gu) && dp_mat(layers[l].down);
        const bool dp_lm = dprecs && dp_mat(lm_head());
        const int ntiles_h = (h + 15) / 16;
        laic::EmbedParams ep{embd.type, embd.q, embd.s, h, embd.nb, d_tokens, d_slots, x, counts, V};
        ep.nseq = nseq;
        if (recs) { ep.rec_out = rec_x; ep.rec_w = layers[0].attn_norm; ep.ss_out = rec_ss; }
        // one sequence with integer records: the row in slices of 256 over several CTAs
        const int ecta = dprecs && L > 0 ? std::max(1, std::min(16, h / 256)) : 1;
        if (dprecs && L > 0) ep.ss_out = rec_ss;
        if (!step_path) {
            t_begin("embed", 0);
            CK(launch_k(laic::embed_kernel, dim3(nseq, ecta), dim3(256), 0, s, pdl, ep));
            ++nl;
            t_end();
        }

        const int nsplit = nsplit_for(nseq);
        last_split = nsplit;
        AttnFn afn = attn_pick(D, G, kv32);
        const size_t kvb = kv32 ? 4 : 2;
        double attn_bytes = 0;
        if (timer)
            for (int i = 0; i < nseq; ++i)
                attn_bytes += (double)(h_pos[h_slots[i]] + 1) * Hkv * D * 2 * kvb + 8.0 * h;

        if (step_path) {  // the whole step (and the lm_head when it shares the layers' type) in one launch
            double wb = 0;
            for (auto& ly : layers) wb += ly.qkv.bytes() + ly.o.bytes() + ly.gu.bytes() + ly.down.bytes();
            if (full && ls_lm) wb += lm_head().bytes();
            t_begin("layers", wb + attn_bytes * L);
            laic::LsParams lp = ls_params(full && ls_lm);
            CK(laic::ls_launch(ls_type, D, G, lp, num_sms(), ls_smem_bytes, s, pdl));
            ++nl;
            t_end();
        }
        for (int l = 0; l < L && !step_path; ++l) {
            Layer& ly = layers[l];
            laic::MvParams p{};
            p.nseq = nseq;
            p.eps = a.rms_eps;
            // qkv
            p.x = x; p.ldx = h; p.norm_w = ly.attn_norm; p.out = q; p.ldo = hq;
            p.q_rows = hq; p.kv_rows = kv; p.head_dim = D; p.rope_pairs = rope_pairs; p.rope_cs = rope_cs;
            p.slots = d_slots; p.pos = pos;
            p.kc = (char*)kc + (size_t)l * kv_layer_stride * kvb;
            p.vc = (char*)vc + (size_t)l * kv_layer_stride * kvb;
            p.kv_slot_stride = kv_slot_stride; p.kv_cap = cap;
            t_begin("qkv", (double)ly.qkv.bytes() + 4.0 * nseq * (h + ly.qkv.rows));
            RecIn r_qkv;
            if (recs || dprecs) {
                r_qkv.xg = rec_x; r_qkv.mode = 1; r_qkv.ss = rec_ss; r_qkv.ss_tiles = l == 0 ? ecta : ntiles_h;
                r_qkv.dp = dprecs;
            }
            CK(launch_matvec(ly.qkv, p, laic::EPI_QKV, kv32, mvs, s, pdl, &nl, &r_qkv, !recs));
            t_end();
            // attention
            laic::AttnParams ap{};
            ap.q = q; ap.ldq = hq; ap.out = attn; ap.ldo = hq;
            ap.kc = p.kc; ap.vc = p.vc; ap.slot_stride = kv_slot_stride; ap.cap = cap;
            ap.heads = H; ap.kv_heads = Hkv; ap.slots = d_slots; ap.pos = pos; ap.nsplit = nsplit;
            ap.part = attn_part; ap.counters = attn_cnt; ap.sqrt_d = sqrtf((float)D); ap.err = mvs.err;
            ap.nseq = nseq; ap.rec_out = recs ? rec_attn : nullptr; ap.nbuf = attn_nbuf(nseq);
            t_begin("attention", attn_bytes);
            if (attn_cluster(nsplit, kv32))
                CK(laic::launch_cluster_k(attn_pick(D, G, kv32, true), dim3(nsplit, Hkv, nseq), dim3(laic::kAttnWarps * 32),
                                          attn_smem(D, kv32, ap.nbuf), s, pdl, nsplit, ap));
            else
                CK(launch_k(afn, dim3(nsplit, Hkv, nseq), dim3(laic::kAttnWarps * 32), attn_smem(D, kv32, ap.nbuf), s,
                            pdl, ap));
            ++nl;
            t_end();
            // o + residual
            laic::MvParams po{};
            po.nseq = nseq; po.x = attn; po.ldx = hq; po.out = x; po.ldo = h;
            RecIn r_o;
            if (recs) {
                po.rec_out = rec_x; po.rec_w = ly.ffn_norm; po.ss_out = rec_ss; r_o.xg = rec_attn; r_o.mode = 2;
            } else if (dprecs) {
                po.ss_out = rec_ss; r_o.mode = 2; r_o.dp = true;
            }
            t_begin("o", (double)ly.o.bytes() + 4.0 * nseq * hq + 8.0 * nseq * h);
            CK(launch_matvec(ly.o, po, residual_epi, kv32, mvs, s, pdl, &nl, &r_o, !recs));
            t_end();
            if (int rc = allreduce_residual(nseq, s, t_begin, t_end, &nl)) return rc;
            // gate/up + swiglu
            laic::MvParams pg{};
            pg.nseq = nseq; pg.eps = a.rms_eps; pg.x = x; pg.ldx = h; pg.norm_w = ly.ffn_norm; pg.out = act; pg.ldo = F;
            RecIn r_gu;
            if (recs || dprecs) {
                r_gu.xg = rec_x; r_gu.mode = 1; r_gu.ss = rec_ss; r_gu.ss_tiles = ntiles_h; r_gu.dp = dprecs;
                if (recs) pg.rec_out = rec_act;
            }
            t_begin("gate_up", (double)ly.gu.bytes() + 4.0 * nseq * (h + F));
            CK(launch_matvec(ly.gu, pg, laic::EPI_SWIGLU, kv32, mvs, s, pdl, &nl, &r_gu, !recs));
            t_end();
            // down + residual
            laic::MvParams pd{};
            pd.nseq = nseq; pd.x = act; pd.ldx = F; pd.out = x; pd.ldo = h;
            RecIn r_dn;
            if (recs || dprecs) {
                r_dn.xg = rec_act; r_dn.mode = 2; r_dn.dp = dprecs;
                pd.ss_out = rec_ss;
                if (recs) {
                    pd.rec_out = rec_x;
                    pd.rec_w = l + 1 < L ? layers[l + 1].attn_norm : out_norm;  // next: QKV, or the lm_head
                }
            }
            t_begin("down", (double)ly.down.bytes() + 4.0 * nseq * (F + 2 * h));
            CK(launch_matvec(ly.down, pd, residual_epi, kv32, mvs, s, pdl, &nl, &r_dn, !recs));
            t_end();
            if (int rc = allreduce_residual(nseq, s, t_begin, t_end, &nl)) return rc;
        }
        if (full) {
            if (!(step_path && ls_lm)) {
                laic::MvParams pl{};
                pl.nseq = nseq; pl.eps = a.rms_eps; pl.x = x; pl.ldx = h; pl.norm_w = out_norm;
                pl.out = tp > 1 ? logits_l : logits; pl.ldo = tp > 1 ? Vl : V;
                t_begin("lm_head", (double)lm_head().bytes() + 4.0 * nseq * (h + Vl));
                RecIn r_lm;
                if ((recs || dp_lm) && L > 0) {
                    r_lm.xg = rec_x; r_lm.mode = 1; r_lm.ss = rec_ss; r_lm.ss_tiles = ntiles_h; r_lm.dp = dp_lm;
                }
                // the lm_head only consumes: the team kernel (its own norm of x) where it is faster
                CK(launch_matvec(lm_head(), pl, laic::EPI_STORE, kv32, mvs, s, pdl, &nl, &r_lm,
                                 !recs || nseq <= LAIC_LM_TEAM_MAX_BATCH));
                t_end();
            }
            if (tp > 1) {  // every rank's vocabulary rows -> logits [nseq][V] on every rank
                t_begin("gather", 4.0 * nseq * V);
                float* dst = nseq == 1 ? logits : logits_g;
                const laic::ncclResult_t r = nccl->AllGather(logits_l, dst, (size_t)nseq * Vl, laic::ncclFloat32, comm, s);
                if (r != laic::ncclSuccess) return fail(LAIC_E_NCCL, std::string("ncclAllGather: ") + nccl->GetErrorString(r));
                if (nseq > 1) {
                    CK(launch_k(laic::gather_logits_kernel, dim3(num_sms()), dim3(256), 0, s, pdl, (const float*)logits_g,
                                logits, tp, nseq, Vl));
                    ++nl;
                }
                t_end();
            }
            laic::SamplerParams sp{logits, V, V, d_slots, counts, d_params, nseq, d_out_ids, d_tokens, pos, d_err,
                                   samp_v, samp_i, samp_cnt};
            // a few sequences: the vocabulary's argmax over several CTAs per sequence
            const int sp_slices = nseq <= 4 ? laic::kSampleSlices : 1;
            t_begin("sampler", (double)nseq * V * 4);
            CK(launch_k(laic::sample_kernel, dim3(nseq, sp_slices), dim3(laic::kSampleThreads), 0, s, pdl, sp));
            ++nl;
            t_end();
            if (mode == MODE_CHAIN)
            {
                CK(launch_k(laic::record_ids_kernel, dim3(1), dim3(256), 0, s, pdl, (const unsigned*)d_out_ids, d_hist,
                            d_hist_count, nseq));
                ++nl;
            } else {
                // the sampled ids and both error flags come back with the step (no extra round trip)
                const int ob = mode == MODE_SPEC1 ? 1 : 0;  // host output buffer
                CK(cudaMemcpyAsync(h_out_ids + (size_t)ob * S, d_out_ids, nseq * sizeof(unsigned), cudaMemcpyDeviceToHost, s));
                CK(cudaMemcpyAsync(h_err + 2 * ob, mvs.err, 4, cudaMemcpyDeviceToHost, s));
                CK(cudaMemcpyAsync(h_err + 2 * ob + 1, d_err, 4, cudaMemcpyDeviceToHost, s));
            }
        } else {
            t_begin("advance", 0);
            CK(launch_k(laic::advance_pos_kernel, dim3(1), dim3(256), 0, s, pdl, (const int*)d_slots, pos, nseq));
            ++nl;
            t_end();
        }
        (full ? launches_step : launches_prefill) = nl;
        return LAIC_OK;
    }

    // Whether one sequence can run as the persistent decode-step kernel: every layer projection
    // Q4_0 (or every one Q8_0), FP16 KV, one GPU, head_dim 64 or 128, at most 8 query heads per
    // kv head, and one CTA per SM with its shared memory. Builds the layer table and
    // the kernel's state (before any capture).
    int prepare_ls() {
        if (ls_checked) return LAIC_OK;
        ls_checked = true;
        ls_ready = false;
        if (!use_ls || kv32 || tp != 1 || (D != 64 && D != 128) || G > 8 || L < 1 || !out_norm) return LAIC_OK;
        const int type = layers[0].qkv.type;
        if (type != T_Q4_0 && type != T_Q8_0) return LAIC_OK;
        for (auto& l : layers)
            if (!l.qkv.q || !l.o.q || !l.gu.q || !l.down.q || l.qkv.type != type || l.o.type != type ||
                l.gu.type != type || l.down.type != type || !l.attn_norm || !l.ffn_norm)
                return LAIC_OK;
        // only on request: per-projection launches measured faster on the 135M-, 1B- and 8B-shaped
        // models (per-phase synchronisation of the one-launch step costs more)
        if (!force_ls) return LAIC_OK;
        const bool lm_in = lm_head().type == type;
        const int nb_max = std::max(std::max(h, hq), F) / 32;
        // the attention chunks of one kv head (at most cap / positions-per-chunk of them) span at
        // most one CTA per chunk: the merge's per-run weights are sized for that
        const int att_runs = std::min(num_sms(), (cap + laic::ls_positions_per_chunk(D) - 1) /
                                                     laic::ls_positions_per_chunk(D));
        int nst = 8;  // attention ring stages (K / V chunks), as many as fit
        size_t smem = 0;
        for (; nst >= 2; --nst)
            if ((smem = laic::ls_smem(type, nst, D, G, nb_max, att_runs)) <= 227 * 1024) break;
        if (nst < 2) return LAIC_OK;
        int bps = 0;
        CK(laic::ls_prepare(type, D, G, smem, &bps));
        if (bps < 1) return LAIC_OK;
        // layer table
        std::vector<laic::LsLayer> tab(L);
        for (int l = 0; l < L; ++l) {
            const Layer& ly = layers[l];
            tab[l] = laic::LsLayer{ly.qkv.q, ly.qkv.s, ly.o.q, ly.o.s, ly.gu.q, ly.gu.s, ly.down.q, ly.down.s,
                                   ly.attn_norm, ly.ffn_norm, (char*)kc + (size_t)l * kv_layer_stride * 2,
                                   (char*)vc + (size_t)l * kv_layer_stride * 2};
        }
        ls_free();
        CK(cudaMalloc(&ls_layers, sizeof(laic::LsLayer) * L));
        CK(cudaMemcpy(ls_layers, tab.data(), sizeof(laic::LsLayer) * L, cudaMemcpyHostToDevice));
        const int Gc = num_sms();
        const int cp = laic::ls_positions_per_chunk(D);
        const int gm = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
        ls_maxch = (cap + cp - 1) / cp;
        CK(cudaMalloc(&ls_rec_x, laic::ls_record_bytes(h / 32)));
        CK(cudaMalloc(&ls_rec_attn, laic::ls_record_bytes(hq / 32)));
        CK(cudaMalloc(&ls_rec_act, laic::ls_record_bytes(F / 32)));
        CK(cudaMalloc(&ls_ss, (size_t)(h / 16) * 4));
        CK(cudaMalloc(&ls_apart, (size_t)Hkv * ls_maxch * gm * (D + 2) * 4));
        ls_done_bytes = (size_t)laic::ls_phases(L) * 8;
        CK(cudaMalloc(&ls_head_tick, (size_t)Hkv * 4));
        CK(cudaMalloc(&ls_done, ls_done_bytes));
        CK(cudaMalloc(&ls_epoch, 8));
        if (trace_on) {
            const size_t tb = ((size_t)Gc * laic::ls_phases(L) * laic::ls_trace_stamps() +
                               (size_t)Gc * laic::ls_trace_warp_words()) * 8;
            CK(cudaMalloc(&ls_trace, tb));
            CK(cudaMemset(ls_trace, 0, tb));
        }
        if (int rc = ls_reset()) return rc;
        ls_type = type;
        ls_nst = nst;
        ls_runs = att_runs;
        ls_smem_bytes = smem;
        ls_lm = lm_in;
        ls_ready = true;
        return LAIC_OK;
    }

    // Counters and tickets of the persistent step kernel back to zero (at set-up, and after a
    // step whose bounded waits ran out and may have left them part-way).
    int ls_reset() {
        if (!ls_done) return LAIC_OK;
        CK(cudaMemset(ls_head_tick, 0, (size_t)Hkv * 4));
        CK(cudaMemset(ls_done, 0, ls_done_bytes));
        CK(cudaMemset(ls_epoch, 0, 8));
        return LAIC_OK;
    }

    void ls_free() {
        void* bufs[] = {ls_layers, ls_rec_x, ls_rec_attn, ls_rec_act, ls_ss, ls_apart, ls_head_tick, ls_done, ls_epoch,
                        ls_trace};
        for (void* b : bufs) if (b) cudaFree(b);
        ls_layers = nullptr; ls_rec_x = ls_rec_attn = ls_rec_act = nullptr; ls_ss = ls_apart = nullptr;
        ls_head_tick = nullptr; ls_done = ls_epoch = nullptr; ls_trace = nullptr;
    }

    laic::LsParams ls_params(bool lm_on) const {
        laic::LsParams lp{};
        lp.layers = ls_layers; lp.L = L;
        lp.h = h; lp.F = F; lp.hq = hq; lp.kv = kv; lp.heads = H; lp.kv_heads = Hkv; lp.rope_pairs = rope_pairs;
        lp.gq = G; lp.eps = a.rms_eps; lp.sqrt_d = sqrtf((float)D);
        lp.emb_type = embd.type; lp.emb_q = embd.q; lp.emb_s = embd.s; lp.emb_nb = embd.nb; lp.vocab = V;
        lp.tokens = d_tokens; lp.slots = d_slots; lp.pos = pos; lp.counts = counts;
        const Mat& lm = lm_head();
        lp.lm_q = lm.q; lp.lm_s = lm.s; lp.lm_rows = lm.rows; lp.lm_on = lm_on ? 1 : 0;
        lp.out_norm = out_norm; lp.logits = logits;
        lp.x = x; lp.q = q; lp.attn = attn; lp.act = act;
        lp.rope_cs = rope_cs; lp.kv_slot_stride = kv_slot_stride; lp.kv_cap = cap;
        lp.rec_x = ls_rec_x; lp.rec_attn = ls_rec_attn; lp.rec_act = ls_rec_act; lp.ss_x = ls_ss;
        lp.apart = ls_apart; lp.att_maxch = ls_maxch; lp.att_runs = ls_runs; lp.head_tick = ls_head_tick;
        lp.done = ls_done; lp.epoch = ls_epoch; lp.err = mvs.err; lp.nstages = ls_nst;
        lp.trace = ls_trace;
        return lp;
    }

    int prefill_alloc() {
        if (pf_x) return LAIC_OK;
        const size_t T = kPfRows;
        size_t wmax = 0, cmax = 0;
        for (auto& l : layers)
            for (const Mat* m : {&l.qkv, &l.o, &l.gu, &l.down}) {
                wmax = std::max(wmax, (size_t)m->rows * m->in);
                cmax = std::max(cmax, (size_t)m->rows);
            }
        const size_t amax = std::max((size_t)std::max(h, hq), (size_t)F);
        CK(cudaMalloc(&pf_x, T * h * 4));
        CK(cudaMalloc(&pf_c, T * cmax * 4));
        CK(cudaMalloc(&pf_q, T * hq * 4));
        CK(cudaMalloc(&pf_attn, T * hq * 4));
        CK(cudaMalloc(&pf_a, T * amax * 2));
        CK(cudaMalloc(&pf_w, wmax * 2));
        CK(cudaMalloc(&pf_slots, T * 4));
        CK(cudaMalloc(&pf_npos, T * 4));
        CK(cudaMalloc(&pf_tokens, T * 4));
        for (auto& l : layers)
            for (const Mat* m : {&l.qkv, &l.o, &l.gu, &l.down})
                pf_ws_bytes = std::max(pf_ws_bytes, laic::gemm_f16_workspace((int)T, m->rows, m->in));
        if (pf_ws_bytes) CK(cudaMalloc(&pf_ws, pf_ws_bytes));
        return LAIC_OK;
    }

    // C[T][rows] = A[T][in] x W^T for one projection (weights dequantised to binary16 first).
    int prefill_gemm(const Mat& m, int T, cudaStream_t s) {
        const int grid = 8 * num_sms();
        laic::dequant_f16_kernel<<<grid, 256, 0, s>>>(m.type, m.q, m.s, m.nb, m.rows, pf_w);
        CK(cudaGetLastError());
        const cudaError_t e = laic::gemm_f16(T, m.rows, m.in, pf_a, pf_w, pf_c, pf_ws, pf_ws_bytes, s);
        if (e != cudaSuccess) return fail(LAIC_E_CUDA, std::string("prefill gemm: ") + cudaGetErrorString(e));
        return LAIC_OK;
    }

    // The prompt tokens of one slot through every layer together (KV cache filled, position
    // advanced, tokens added to the slot's history), like n prefill steps.
    int prefill_batch(int slot, const uint32_t* tokens, int n) {
        if (int rc = prefill_alloc()) return rc;
        cudaStream_t s = st;
        const int grid = 8 * num_sms();
        const size_t kvb = 2;
        for (int t0 = 0; t0 < n; t0 += kPfRows) {
            const int T = std::min(kPfRows, n - t0);
            const int p0 = (int)h_pos[slot];
            CK(cudaMemcpyAsync(pf_tokens, tokens + t0, (size_t)T * 4, cudaMemcpyHostToDevice, s));
            laic::prefill_rows_kernel<<<(T + 255) / 256, 256, 0, s>>>(slot, p0, T, pf_slots, pf_npos);
            laic::EmbedParams ep{embd.type, embd.q, embd.s, h, embd.nb, pf_tokens, pf_slots, pf_x, counts, V};
            laic::embed_kernel<<<T, 256, 0, s>>>(ep);
            CK(cudaGetLastError());
            for (int l = 0; l < L; ++l) {
                Layer& ly = layers[l];
                __half* kcl = (__half*)((char*)kc + ((size_t)l * kv_layer_stride + (size_t)slot * kv_slot_stride) * kvb);
                __half* vcl = (__half*)((char*)vc + ((size_t)l * kv_layer_stride + (size_t)slot * kv_slot_stride) * kvb);
                // qkv
                laic::rmsnorm_f16_kernel<<<T, 256, 0, s>>>(pf_x, h, ly.attn_norm, a.rms_eps, h, pf_a, h);
                if (int rc = prefill_gemm(ly.qkv, T, s)) return rc;
                laic::QkvPostParams qp{pf_c, T, hq, kv, D, rope_pairs, p0, rope_cs, pf_q, kcl, vcl, cap};
                laic::qkv_post_kernel<<<grid, 256, 0, s>>>(qp);
                // attention: one query row per token, causal through its own position
                laic::AttnParams ap{};
                ap.q = pf_q; ap.ldq = hq; ap.out = pf_attn; ap.ldo = hq;
                ap.kc = (char*)kc + (size_t)l * kv_layer_stride * kvb; ap.vc = (char*)vc + (size_t)l * kv_layer_stride * kvb;
                ap.slot_stride = kv_slot_stride; ap.cap = cap; ap.heads = H; ap.kv_heads = Hkv;
                ap.slots = pf_slots; ap.pos = pos; ap.npos = pf_npos; ap.nsplit = 1;
                ap.part = attn_part; ap.counters = attn_cnt; ap.sqrt_d = sqrtf((float)D); ap.err = mvs.err; ap.nseq = T;
                CK(laic::launch_k(attn_pick(D, G, false), dim3(1, Hkv, T), dim3(laic::kAttnWarps * 32), attn_smem(D, false),
                                  s, false, ap));
                // o + residual
                laic::to_f16_kernel<<<grid, 256, 0, s>>>(pf_attn, pf_a, (size_t)T * hq);
                if (int rc = prefill_gemm(ly.o, T, s)) return rc;
                laic::residual_add_kernel<<<grid, 256, 0, s>>>(pf_x, pf_c, (size_t)T * h);
                // gate/up + swiglu, down + residual
                laic::rmsnorm_f16_kernel<<<T, 256, 0, s>>>(pf_x, h, ly.ffn_norm, a.rms_eps, h, pf_a, h);
                if (int rc = prefill_gemm(ly.gu, T, s)) return rc;
                laic::swiglu_f16_kernel<<<grid, 256, 0, s>>>(pf_c, T, F, pf_a);
                if (int rc = prefill_gemm(ly.down, T, s)) return rc;
                laic::residual_add_kernel<<<grid, 256, 0, s>>>(pf_x, pf_c, (size_t)T * h);
                CK(cudaGetLastError());
            }
            laic::add_pos_kernel<<<1, 32, 0, s>>>(pos, slot, T);
            CK(cudaGetLastError());
            CK(cudaStreamSynchronize(s));  // the token buffer is reused by the next pass
            h_pos[slot] += T;
        }
        return LAIC_OK;
    }

    // Size the matvec scratch for `nseq` sequences (before any capture).
    int reserve_scratch(int nseq) {
        if (int rc = prepare_ls()) return rc;
        MvNeed need;
        auto see = [&](const Mat& m) {
            if (m.q) need.merge(mv_need(m, nseq));
        };
        for (auto& l : layers) { see(l.qkv); see(l.o); see(l.gu); see(l.down); }
        see(lm_head());
        bool moved = false;
        int rc = mv_scratch_reserve(mvs, need, &moved);
        if (!rc && moved) {  // graphs captured the old buffers
            for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
            graphs.clear();
        }
        return rc;
    }

    int run(int nseq, int mode) {
        int rc0 = reserve_scratch(nseq);
        if (rc0) return rc0;
        if (!use_graph) return enqueue(nseq, mode, st, nullptr);
        auto key = std::make_pair(nseq, mode);
        auto it = graphs.find(key);
        if (it == graphs.end()) {
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            int rc = enqueue(nseq, mode, st, nullptr);
            cudaError_t ce = cudaStreamEndCapture(st, &g);
            if (rc) { if (g) cudaGraphDestroy(g); return rc; }
            if (ce != cudaSuccess) return fail(LAIC_E_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
            cudaGraphExec_t ex = nullptr;
            ce = cudaGraphInstantiate(&ex, g, 0);
            cudaGraphDestroy(g);
            if (ce != cudaSuccess) return fail(LAIC_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
            it = graphs.emplace(key, ex).first;
        }
        CK(cudaGraphLaunch(it->second, st));
        return LAIC_OK;
    }

    int check_batch(int nseq, const uint32_t* tokens, const int32_t* slots) {
        if (nseq <= 0 || nseq > S) return fail(LAIC_E_INVALID, "nseq must be in [1, max_seqs]");
        if (!tokens || !slots) return fail(LAIC_E_INVALID, "null tokens or slots");
        std::string missing;
        if (!ready(missing)) return fail(LAIC_E_MISSING, "missing tensor: " + missing);
        std::vector<char> seen(S, 0);
        for (int i = 0; i < nseq; ++i) {
            if (slots[i] < 0 || slots[i] >= S) return fail(LAIC_E_INVALID, "slot out of range");
            if (seen[slots[i]]) return fail(LAIC_E_INVALID, "slot listed twice in one step");
            seen[slots[i]] = 1;
            if (tokens[i] >= (uint32_t)V || tokens[i] >= (uint32_t)embd.rows) return fail(LAIC_E_INVALID, "invalid embedding tensor");
            if (h_pos[slots[i]] >= cap) return fail(LAIC_E_CONTEXT, "context length exceeded");
        }
        return LAIC_OK;
    }
};

namespace {

int parse_layer(const std::string& name, int& layer, std::string& part) {
    if (name.rfind("blk.", 0) != 0) return 0;
    size_t dot = name.find('.', 4);
    if (dot == std::string::npos) return 0;
    try { layer = std::stoi(name.substr(4, dot - 4)); } catch (...) { return 0; }
    std::string rest = name.substr(dot + 1);
    const std::string suf = ".weight";
    if (rest.size() <= suf.size() || rest.compare(rest.size() - suf.size(), suf.size(), suf) != 0) return 0;
    part = rest.substr(0, rest.size() - suf.size());
    return 1;
}

int upload_norm(float** dst, int type, const void* data, size_t n, size_t nbytes) {
    if (type != T_F32 && type != T_F16) return fail(LAIC_E_UNSUPPORTED, "norm weights must be F32 or F16");
    if (nbytes < elem_bytes(type, n)) return fail(LAIC_E_INVALID, "tensor data out of range");
    std::vector<float> v(n);
    if (type == T_F32) std::memcpy(v.data(), data, n * 4);
    else {
        const uint16_t* hsrc = (const uint16_t*)data;
        for (size_t i = 0; i < n; ++i) {
            __half_raw r; r.x = hsrc[i];
            v[i] = __half2float(__half(r));
        }
    }
    if (!*dst) CK(cudaMalloc(dst, n * 4));
    CK(cudaMemcpy(*dst, v.data(), n * 4, cudaMemcpyHostToDevice));
    return LAIC_OK;
}

}  // namespace

extern "C" {

const char* laic_last_error(void) { return g_err.c_str(); }

int laic_dev_create(const laic_dev_desc* desc, const laic_dev_opts* opts, laic_dev** out) {
    if (!desc || !out) return fail(LAIC_E_INVALID, "null argument");
    *out = nullptr;
    laic_dev_opts o{};
    o.max_seqs = 1; o.tp_size = 1;
    if (opts) o = *opts;
    const laic_dev_desc& a = *desc;
    const int tp = std::max(1, o.tp_size);
    if (tp > 1) {
        if (tp > 8) return fail(LAIC_E_UNSUPPORTED, "tp_size must be at most 8 (one node)");
        if (o.tp_rank < 0 || o.tp_rank >= tp) return fail(LAIC_E_INVALID, "tp_rank out of range");
        if (!o.nccl_id) return fail(LAIC_E_INVALID, "tp_size > 1 needs nccl_id (laic_nccl_unique_id on rank 0)");
        if (!a.heads || !a.kv_heads || a.heads % tp || a.kv_heads % tp)
            return fail(LAIC_E_UNSUPPORTED, "heads and kv_heads must be multiples of tp_size");
        if (a.ffn % (32 * (uint32_t)tp)) return fail(LAIC_E_UNSUPPORTED, "ffn / tp_size must be a multiple of 32");
        if (a.vocab % tp) return fail(LAIC_E_UNSUPPORTED, "vocab must be a multiple of tp_size");
    }
    if (!a.hidden || !a.layers || !a.heads || !a.kv_heads || a.hidden % a.heads || a.heads % a.kv_heads || !a.ffn || !a.vocab)
        return fail(LAIC_E_INVALID, "invalid llama architecture metadata");
    const uint32_t D = a.hidden / a.heads;
    const uint32_t rd = a.rope_dim ? a.rope_dim : D;
    if (!rd || rd > D || (rd & 1)) return fail(LAIC_E_INVALID, "invalid RoPE dimension");
    if (D != 32 && D != 64 && D != 128) return fail(LAIC_E_UNSUPPORTED, "head_dim must be 32, 64 or 128");
    if (a.heads / a.kv_heads > 8) return fail(LAIC_E_UNSUPPORTED, "at most 8 query heads per kv head");
    if (a.hidden % 32 || a.ffn % 32) return fail(LAIC_E_UNSUPPORTED, "hidden and ffn must be multiples of 32");
    if (o.max_seqs < 1) return fail(LAIC_E_INVALID, "max_seqs must be >= 1");
    if (o.max_seqs > 64) return fail(LAIC_E_UNSUPPORTED, "at most 64 sequence slots per device");
    const uint32_t ctx = a.ctx ? a.ctx : 2048;
    int cap = o.kv_capacity > 0 ? std::min<int>(o.kv_capacity, (int)ctx) : (int)ctx;

    CK(cudaSetDevice(o.device));
    std::unique_ptr<laic_dev> d(new laic_dev());
    d->a = a; d->a.ctx = ctx; d->a.rope_dim = rd;
    d->o = o; d->device = o.device;
    d->tp = tp; d->tr = tp > 1 ? o.tp_rank : 0;
    d->H = a.heads / tp; d->Hkv = a.kv_heads / tp; d->D = D; d->G = a.heads / a.kv_heads; d->h = a.hidden;
    d->kv = d->Hkv * D; d->hq = d->H * D; d->F = a.ffn / tp; d->V = a.vocab; d->Vl = a.vocab / tp;
    d->L = a.layers; d->S = o.max_seqs; d->cap = cap;
    d->rope_pairs = rd / 2;
    d->kv32 = (o.flags & LAIC_FLAG_KV_F32) != 0;
    d->use_graph = !(o.flags & LAIC_FLAG_NO_GRAPH);
    d->use_pdl = !(o.flags & LAIC_FLAG_NO_PDL);
    d->use_ls = (o.flags & LAIC_FLAG_LAYER_LAUNCHES) == 0;
    d->force_ls = (o.flags & LAIC_FLAG_STEP_KERNEL) != 0;
    d->q4_upstream = (o.flags & LAIC_FLAG_Q4_0_UPSTREAM) != 0;
    d->use_spec = (o.flags & LAIC_FLAG_NO_SPECULATION) == 0;
    d->trace_on = (o.flags & LAIC_FLAG_TRACE) != 0;
    d->layers.resize(a.layers);
    d->h_pos.assign(o.max_seqs, 0);
    CK(cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking));
    // set kernel attributes now: graph capture must not see attribute calls
    CK(laic::mv_set_attributes());
    if (!d->kv32)
        for (bool cl : {false, true})
            CK(cudaFuncSetAttribute(attn_pick(D, d->G, false, cl), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)attn_smem(D, false, attn_max_nbuf(D))));

    const size_t S = o.max_seqs, kvb = d->kv32 ? 4 : 2;
    CK(cudaMalloc(&d->x, S * d->h * 4));
    CK(cudaMalloc(&d->q, S * d->hq * 4));
    CK(cudaMalloc(&d->attn, S * d->hq * 4));
    CK(cudaMalloc(&d->act, S * d->F * 4));
    CK(cudaMalloc(&d->logits, S * d->V * 4));
    if (tp > 1) {
        CK(cudaMalloc(&d->logits_l, S * d->Vl * 4));
        CK(cudaMalloc(&d->logits_g, S * d->V * 4));
        std::string why;
        d->nccl = laic::nccl_api(why);
        if (!d->nccl) return fail(LAIC_E_NCCL, why);
        laic::ncclUniqueId id;
        std::memcpy(&id, o.nccl_id, sizeof id);
        const laic::ncclResult_t r = d->nccl->CommInitRank(&d->comm, tp, id, d->tr);
        if (r != laic::ncclSuccess) return fail(LAIC_E_NCCL, std::string("ncclCommInitRank: ") + d->nccl->GetErrorString(r));
        d->ar.err = nullptr;
    }
    d->kv_slot_stride = (long long)d->Hkv * cap * D;
    d->kv_layer_stride = d->kv_slot_stride * (long long)S;
    const size_t kv_bytes = (size_t)d->kv_layer_stride * d->L * kvb;
    CK(cudaMalloc(&d->kc, kv_bytes));
    CK(cudaMalloc(&d->vc, kv_bytes));
    CK(cudaMemset(d->kc, 0, kv_bytes));
    CK(cudaMemset(d->vc, 0, kv_bytes));
    CK(cudaMalloc(&d->pos, S * 4));
    CK(cudaMemset(d->pos, 0, S * 4));
    if (d->tile_step(S) || d->tp == 1) {  // activation records between the projections
        CK(cudaMalloc(&d->rec_x, S * d->h * 4));
        CK(cudaMalloc(&d->rec_act, S * d->F * 4));
        CK(cudaMalloc(&d->rec_attn, S * d->hq * 4));
        CK(cudaMalloc(&d->rec_ss, S * ((d->h + 15) / 16) * 4));
    }
    CK(cudaMalloc(&d->counts, S * d->V * 4));
    CK(cudaMemset(d->counts, 0, S * d->V * 4));

    // RoPE table with the reference's float arithmetic (src/inference_v2.cpp:25):
    // a = float(pos) * pow(theta, -float(i)/float(head_dim)), (cos a, sin a)
    std::vector<float2> cs((size_t)cap * d->rope_pairs);
    const float theta = a.rope_theta > 0 ? a.rope_theta : 10000.f;
    for (int p = 0; p < cap; ++p)
        for (int j = 0; j < d->rope_pairs; ++j) {
            const int i = 2 * j;
            const float ang = float(p) * std::pow(theta, -float(i) / float(D));
            cs[(size_t)p * d->rope_pairs + j] = make_float2(std::cos(ang), std::sin(ang));
        }
    CK(cudaMalloc(&d->rope_cs, std::max<size_t>(1, cs.size()) * sizeof(float2)));
    if (!cs.empty()) CK(cudaMemcpy(d->rope_cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice));

    d->max_split = std::max(1, std::min(64, (cap + 31) / 32));
    CK(cudaMalloc(&d->attn_part, S * d->Hkv * d->max_split * d->G * (D + 2) * 4));
    CK(cudaMalloc(&d->attn_cnt, S * d->Hkv * 4));
    CK(cudaMemset(d->attn_cnt, 0, S * d->Hkv * 4));

    CK(cudaMalloc(&d->d_tokens, S * 4));
    CK(cudaMalloc(&d->d_out_ids, S * 4));
    CK(cudaMalloc(&d->d_slots, S * 4));
    CK(cudaMalloc(&d->d_err, 4));
    CK(cudaMemset(d->d_err, 0, 4));
    CK(cudaMalloc(&d->samp_v, S * laic::kSampleSlices * 4));
    CK(cudaMalloc(&d->samp_i, S * laic::kSampleSlices * 4));
    CK(cudaMalloc(&d->samp_cnt, S * 4));
    CK(cudaMemset(d->samp_cnt, 0, S * 4));
    CK(cudaMalloc(&d->d_hist_count, 4));
    CK(cudaMalloc(&d->d_params, S * sizeof(laic::SampleDev)));
    CK(cudaMallocHost(&d->h_tokens, S * 4));
    CK(cudaMallocHost(&d->h_out_ids, 2 * S * 4));
    CK(cudaMallocHost(&d->h_err, 4 * sizeof(int)));
    CK(cudaEventCreateWithFlags(&d->spec_ev[0], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&d->spec_ev[1], cudaEventDisableTiming));
    CK(cudaMallocHost(&d->h_spec, 2 * (size_t)o.max_seqs * sizeof(int)));
    CK(cudaMalloc(&d->d_spec, 2 * (size_t)o.max_seqs * sizeof(int)));
    d->h_err[0] = d->h_err[1] = d->h_err[2] = d->h_err[3] = 0;
    CK(cudaMallocHost(&d->h_slots, S * 4));
    CK(cudaMallocHost(&d->h_params, S * sizeof(laic::SampleDev)));
    if (tp > 1) {
        // the residual allreduce through peer memory unless LAIC_TP_NCCL_ALLREDUCE=1 asks for NCCL
        const char* env = std::getenv("LAIC_TP_NCCL_ALLREDUCE");
        if (!(env && env[0] == '1')) {
            if (int rc = mv_scratch_reserve(d->mvs, MvNeed{})) return rc;  // the error flag
            if (int rc = d->setup_p2p_allreduce()) return rc;
            d->ar.err = d->mvs.err;
        }
    }
    CK(cudaDeviceSynchronize());
    *out = d.release();
    return LAIC_OK;
}

void laic_dev_destroy(laic_dev* d) {
    if (!d) return;
    cudaSetDevice(d->device);
    cudaStreamSynchronize(d->st);
    for (cudaEvent_t ev : d->spec_ev) if (ev) cudaEventDestroy(ev);
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);  // graphs holding NCCL calls go first
    d->graphs.clear();
    for (int q = 0; q < d->tp && d->ar_p2p; ++q) {
        if (q == d->tr) continue;
        if (d->ar.box[q]) cudaIpcCloseMemHandle(d->ar.box[q]);
        if (d->ar.flags[q]) cudaIpcCloseMemHandle(d->ar.flags[q]);
    }
    if (d->comm) d->nccl->CommDestroy(d->comm);
    for (auto& l : d->layers) {
        mat_free(l.qkv); mat_free(l.o); mat_free(l.gu); mat_free(l.down);
        if (l.attn_norm) cudaFree(l.attn_norm);
        if (l.ffn_norm) cudaFree(l.ffn_norm);
    }
    mat_free(d->embd); mat_free(d->lm);
    mv_scratch_free(d->mvs);
    d->ls_free();
    void* bufs[] = {d->out_norm, d->x, d->q, d->attn, d->act, d->logits, d->kc, d->vc, d->pos, d->counts,
                    d->rope_cs, d->attn_part, d->attn_cnt, d->d_tokens, d->d_out_ids, d->d_slots, d->d_err, d->d_params,
                    d->d_hist, d->d_hist_count, d->logits_l, d->logits_g, d->rec_x, d->rec_act, d->rec_ss, d->rec_attn,
                    d->ar_box, d->ar_flags, d->ar_ctr,
                    d->pf_x, d->pf_c, d->pf_q, d->pf_attn, d->pf_a, d->pf_w, d->pf_slots, d->pf_npos, d->pf_tokens,
                    d->pf_ws, d->samp_v, d->samp_i, d->samp_cnt, d->d_spec};
    for (void* b : bufs) if (b) cudaFree(b);
    if (d->h_spec) cudaFreeHost(d->h_spec);
    void* hb[] = {d->h_tokens, d->h_out_ids, d->h_slots, d->h_params, d->h_err};
    for (void* b : hb) if (b) cudaFreeHost(b);
    if (d->st) cudaStreamDestroy(d->st);
    delete d;
}

int laic_dev_upload(laic_dev* d, const char* cname, int32_t type, const uint64_t* shape, int32_t ndim,
                    const void* data, size_t nbytes) {
    if (!d || !cname || !shape || !data) return fail(LAIC_E_INVALID, "null argument");
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    const std::string name(cname);
    size_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= shape[i];
    if (nbytes < elem_bytes(type, n)) return fail(LAIC_E_INVALID, "tensor data out of range: " + name);
    std::vector<uint8_t> conv;  // blocks held as another type with the same values (convert_blocks)
    int ctype = type;
    if (convert_blocks(type, (const uint8_t*)data, n / 32, d->q4_upstream, &ctype, conv)) {
        type = ctype;
        data = conv.data();
        nbytes = conv.size();
    }
    auto shape_is = [&](uint64_t in, uint64_t out) { return ndim == 2 && shape[0] == in && shape[1] == out; };
    // any graph captured before this upload points at old buffers
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    d->graphs.clear();
    d->ls_checked = false;

    if (name == "output_norm.weight") {
        if (n != (size_t)d->h) return fail(LAIC_E_INVALID, "invalid norm tensor: " + name);
        int rc = upload_norm(&d->out_norm, type, data, n, nbytes);
        if (!rc) d->have_onorm = true;
        return rc;
    }
    if (name == "token_embd.weight" || name == "output.weight") {
        const bool is_embd = name == "token_embd.weight";
        if (ndim != 2 || shape[0] != (uint64_t)d->h) return fail(LAIC_E_INVALID, "unexpected weight shape: " + name);
        if (!is_embd && shape[1] != (uint64_t)d->V) return fail(LAIC_E_INVALID, "unexpected weight shape: " + name);
        if (d->tp > 1 && (is_embd ? !d->have_out : true)) {
            // this rank's lm_head rows (the output matrix, or the tied embedding until one arrives)
            if (is_embd && shape[1] != (uint64_t)d->V) return fail(LAIC_E_INVALID, "unexpected weight shape: " + name);
            mat_free(d->lm);
            int rc = mat_alloc(d->lm, type, d->Vl, d->h);
            if (rc) return rc;
            const size_t rb = elem_bytes(type, (size_t)d->h);
            rc = mat_fill(d->lm, (const uint8_t*)data + (size_t)d->tr * d->Vl * rb, d->Vl, 1, 0, d->st);
            if (rc) return rc;
            d->have_lm = true;
            if (!is_embd) { d->have_out = true; return LAIC_OK; }
        }
        Mat& m = is_embd ? d->embd : d->lm;
        mat_free(m);
        int rc = mat_alloc(m, type, (int)shape[1], d->h);
        if (rc) return rc;
        rc = mat_fill(m, (const uint8_t*)data, (int)shape[1], 1, 0, d->st);
        if (rc) return rc;
        if (is_embd) d->have_embd = true; else d->have_out = true;
        return LAIC_OK;
    }
    int l;
    std::string part;
    if (!parse_layer(name, l, part) || l < 0 || l >= d->L) return LAIC_OK;  // not used by the decode path
    Layer& ly = d->layers[l];
    // h: hidden; hq, kv, F: this rank's query width, kv width and ffn rows; *_full: the GGUF's
    const int h = d->h, kv = d->kv, F = d->F, hq = d->hq, tr = d->tr;
    const int kv_full = (int)d->a.kv_heads * d->D, F_full = (int)d->a.ffn;
    const uint8_t* src = (const uint8_t*)data;
    // rows [r0, ...) of a [rows][in] tensor; columns [c0, c0 + nc) of each row gathered on the host
    auto rows_from = [&](int r0, int in) { return src + (size_t)r0 * elem_bytes(type, (size_t)in); };
    std::vector<uint8_t> colbuf;
    auto cols_of = [&](int rows, int in, int c0, int nc) -> const uint8_t* {
        if (c0 == 0 && nc == in) return src;
        const size_t rb = elem_bytes(type, (size_t)in), cb = elem_bytes(type, (size_t)nc), ob = elem_bytes(type, (size_t)c0);
        colbuf.resize((size_t)rows * cb);
        for (int r = 0; r < rows; ++r) std::memcpy(colbuf.data() + (size_t)r * cb, src + (size_t)r * rb + ob, cb);
        return colbuf.data();
    };
    auto ensure = [&](Mat& m, int rows, int in) -> int {
        if (m.q && m.type != type) return fail(LAIC_E_UNSUPPORTED, "fused projections need one type: " + name);
        if (!m.q) return mat_alloc(m, type, rows, in);
        return LAIC_OK;
    };
    int rc = LAIC_OK;
    if (part == "attn_norm" || part == "ffn_norm") {
        if (n != (size_t)h) return fail(LAIC_E_INVALID, "invalid norm tensor: " + name);
        const bool an = part == "attn_norm";
        rc = upload_norm(an ? &ly.attn_norm : &ly.ffn_norm, type, data, n, nbytes);
        if (!rc) ly.have |= an ? H_ANORM : H_FNORM;
    } else if (part == "attn_q" || part == "attn_k" || part == "attn_v") {
        const bool isq = part == "attn_q";
        if (!shape_is(h, isq ? h : kv_full)) return fail(LAIC_E_INVALID, "unexpected weight shape: " + name);
        if ((rc = ensure(ly.qkv, hq + 2 * kv, h))) return rc;
        const int out = isq ? hq : kv;  // this rank's heads: rows [tr * out, (tr + 1) * out)
        const long long off = isq ? 0 : part == "attn_k" ? hq : hq + kv;
        rc = mat_fill(ly.qkv, rows_from(tr * out, h), out, 1, off, d->st);
        if (!rc) ly.have |= isq ? H_Q : part == "attn_k" ? H_K : H_V;
    } else if (part == "attn_output") {
        if (!shape_is(h, h)) return fail(LAIC_E_INVALID, "unexpected weight shape: " + name);
        if ((rc = ensure(ly.o, h, hq))) return rc;
        rc = mat_fill(ly.o, cols_of(h, h, tr * hq, hq), h, 1, 0, d->st);  // columns of this rank's heads
        if (!rc) ly.have |= H_O;
    } else if (part == "ffn_gate" || part == "ffn_up") {
        if (!shape_is(h, F_full)) return fail(LAIC_E_INVALID, "unexpected weight shape: " + name);
        if ((rc = ensure(ly.gu, 2 * F, h))) return rc;
        rc = mat_fill(ly.gu, rows_from(tr * F, h), F, 2, part == "ffn_gate" ? 0 : 1, d->st);
        if (!rc) ly.have |= part == "ffn_gate" ? H_GATE : H_UP;
    } else if (part == "ffn_down") {
        if (!shape_is(F_full, h)) return fail(LAIC_E_INVALID, "unexpected weight shape: " + name);
        if ((rc = ensure(ly.down, h, F))) return rc;
        rc = mat_fill(ly.down, cols_of(h, F_full, tr * F, F), h, 1, 0, d->st);  // this rank's ffn columns
        if (!rc) ly.have |= H_DOWN;
    }
    return rc;
}

static int fill_inputs(laic_dev* d, int32_t nseq, const uint32_t* tokens, const int32_t* slots) {
    int rc = d->check_batch(nseq, tokens, slots);
    if (rc) return rc;
    std::memcpy(d->h_tokens, tokens, nseq * 4);
    std::memcpy(d->h_slots, slots, nseq * 4);
    return LAIC_OK;
}

int laic_dev_prefill_batch(laic_dev* d, int32_t slot, const uint32_t* tokens, int32_t n) {
    if (!d || !tokens) return fail(LAIC_E_INVALID, "null argument");
    if (n < 0) return fail(LAIC_E_INVALID, "negative token count");
    if (n == 0) return LAIC_OK;
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    if (slot < 0 || slot >= d->S) return fail(LAIC_E_INVALID, "slot out of range");
    std::string missing;
    if (!d->ready(missing)) return fail(LAIC_E_MISSING, "missing tensor: " + missing);
    for (int i = 0; i < n; ++i)
        if (tokens[i] >= (uint32_t)d->V || tokens[i] >= (uint32_t)d->embd.rows)
            return fail(LAIC_E_INVALID, "invalid embedding tensor");
    if (d->h_pos[slot] + n > d->cap) return fail(LAIC_E_CONTEXT, "context length exceeded");
    if (d->kv32 || d->tp > 1 || !(d->D == 32 || d->D == 64 || d->D == 128)) {
        // FP32-KV parity mode and tensor parallel runs: the per-token steps
        for (int i = 0; i < n; ++i) {
            const int32_t sl = slot;
            if (int rc = laic_dev_prefill(d, 1, tokens + i, &sl)) return rc;
        }
        return LAIC_OK;
    }
    return d->prefill_batch(slot, tokens, n);
}

int laic_dev_prefill(laic_dev* d, int32_t nseq, const uint32_t* tokens, const int32_t* slots) {
    if (!d) return fail(LAIC_E_INVALID, "null device");
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    int rc = fill_inputs(d, nseq, tokens, slots);
    if (rc) return rc;
    if ((rc = d->run(nseq, MODE_PREFILL))) return rc;
    CK(cudaStreamSynchronize(d->st));
    for (int i = 0; i < nseq; ++i) d->h_pos[slots[i]] += 1;
    return LAIC_OK;
}

static double canonical_draw(uint64_t seed) {
    std::mt19937_64 rng(seed ? seed : std::random_device{}());
    return std::generate_canonical<double, std::numeric_limits<double>::digits>(rng);
}

static int fill_params(laic_dev* d, int32_t nseq, const laic_sample_params* params, int32_t nparams) {
    laic_sample_params greedy{0.f, 0, 1.f, 1.f, 0};
    if (!params) { params = &greedy; nparams = 1; }
    if (nparams != 1 && nparams != nseq) return fail(LAIC_E_INVALID, "nparams must be 1 or nseq");
    for (int i = 0; i < nseq; ++i) {
        const laic_sample_params& sp = params[nparams == 1 ? 0 : i];
        laic::SampleDev& o = d->h_params[i];
        o.temperature = sp.temperature; o.top_k = sp.top_k; o.top_p = sp.top_p; o.repeat_penalty = sp.repeat_penalty;
        // the reference re-seeds mt19937_64 on every sample() call: one canonical draw per call
        o.u = sp.temperature > 0.f ? canonical_draw(sp.seed) : 0.0;
    }
    return LAIC_OK;
}

// The message of a bounded device wait that ran out (the codes of common.cuh).
static std::string wait_error_text(int code) {
    switch (code) {
    case laic::kErrMbarrier: return "device wait timed out: a bulk copy into shared memory never completed";
    case laic::kErrTeamMerge: return "device wait timed out: a matvec warp team's partial-sum slot was never released";
    case laic::kErrGridBarrier: return "device wait timed out: a decode-step grid barrier was not reached by every CTA";
    case laic::kErrPeerFlag: return "device wait timed out: a tensor-parallel peer never published its allreduce slice";
    case laic::kErrDepCounter: return "device wait timed out: a decode-step dependency counter never reached its target";
    }
    return "device wait timed out (code " + std::to_string(code) + ")";
}

// After a synchronised MODE_STEP run: the error flags its graph copied to pinned memory.
static int check_step_err(laic_dev* d, int buf = 0) {
    const int mv_err = d->h_err[2 * buf], sample_err = d->h_err[2 * buf + 1];
    if (mv_err) {
        CK(cudaMemset(d->mvs.err, 0, 4));
        d->h_err[2 * buf] = 0;
        if (int rc = d->ls_reset()) return rc;
        return fail(LAIC_E_CUDA, wait_error_text(mv_err));
    }
    if (sample_err) {
        CK(cudaMemset(d->d_err, 0, 4));
        d->h_err[2 * buf + 1] = 0;
        return fail(LAIC_E_UNSUPPORTED, "sampling request needs more than 1024 candidates (top_k or top_p mass)");
    }
    return LAIC_OK;
}

static int check_sampler_err(laic_dev* d) {
    int err = 0;
    if (d->mvs.err) {
        CK(cudaMemcpy(&err, d->mvs.err, 4, cudaMemcpyDeviceToHost));
        if (err) {
            CK(cudaMemset(d->mvs.err, 0, 4));
            if (int rc = d->ls_reset()) return rc;
            return fail(LAIC_E_CUDA, wait_error_text(err));
        }
    }
    CK(cudaMemcpy(&err, d->d_err, 4, cudaMemcpyDeviceToHost));
    if (err) {
        CK(cudaMemset(d->d_err, 0, 4));
        return fail(LAIC_E_UNSUPPORTED, "sampling request needs more than 1024 candidates (top_k or top_p mass)");
    }
    return LAIC_OK;
}

int laic_dev_step(laic_dev* d, int32_t nseq, const uint32_t* tokens, const int32_t* slots,
                  const laic_sample_params* params, int32_t nparams, uint32_t* out_ids, float* out_logits) {
    if (!d) return fail(LAIC_E_INVALID, "null device");
    CK(cudaSetDevice(d->device));
    int rc = fill_inputs(d, nseq, tokens, slots);
    if (rc == LAIC_OK) rc = fill_params(d, nseq, params, nparams);
    if (rc) {
        if (int rc2 = d->spec_cancel()) return rc2;
        return rc;
    }
    // this call feeds back the previous step's sampled ids (same slots and parameters)?
    bool feedback = nseq == d->last_nseq;
    for (int i = 0; feedback && i < nseq; ++i) {
        const laic::SampleDev &a = d->h_params[i], &b = d->last_params[i];
        feedback = slots[i] == d->last_slots[i] && tokens[i] == d->last_ids[i] && a.temperature == b.temperature &&
                   a.top_k == b.top_k && a.top_p == b.top_p && a.repeat_penalty == b.repeat_penalty && a.u == b.u;
    }
    // room for a further guess after this step: every slot one position below the capacity
    bool room = true;
    for (int i = 0; i < nseq; ++i) room = room && d->h_pos[slots[i]] + 1 < d->cap;
    const bool guess = d->use_spec && feedback && d->tp == 1;
    int buf = 0;  // host output buffer of this call's step
    if (d->spec_pending && feedback) {
        // the pending guess is this call's step: queue the following guess behind it before
        // waiting, so the stream never drains while the caller keeps feeding back its ids
        d->spec_pending = false;
        buf = d->spec_buf;
        if (out_logits)  // (in stream order, before the next guess overwrites them)
            CK(cudaMemcpyAsync(out_logits, d->logits, (size_t)nseq * d->V * 4, cudaMemcpyDeviceToHost, d->st));
        const bool next = guess && room;
        if (next) {
            if ((rc = d->run(nseq, buf ? MODE_SPEC0 : MODE_SPEC1))) return rc;
            CK(cudaEventRecord(d->spec_ev[buf ^ 1], d->st));
        }
        CK(cudaEventSynchronize(d->spec_ev[buf]));
        d->spec_pending = next;
        d->spec_buf = buf ^ 1;
    } else {
        if ((rc = d->spec_cancel())) return rc;
        if ((rc = d->run(nseq, MODE_STEP))) return rc;
        if (out_logits)
            CK(cudaMemcpyAsync(out_logits, d->logits, (size_t)nseq * d->V * 4, cudaMemcpyDeviceToHost, d->st));
        CK(cudaStreamSynchronize(d->st));
        if (guess && room) {  // the first guess of a feedback loop (buffer 1: this step's outputs are in 0)
            if ((rc = d->run(nseq, MODE_SPEC1))) return rc;
            CK(cudaEventRecord(d->spec_ev[1], d->st));
            d->spec_pending = true;
            d->spec_buf = 1;
        }
    }
    for (int i = 0; i < nseq; ++i) d->h_pos[slots[i]] += 1;
    if ((rc = check_step_err(d, buf))) {
        if (int rc2 = d->spec_cancel()) return rc2;  // (the guess behind a failed step is not kept)
        d->last_nseq = 0;
        return rc;
    }
    const unsigned* ids = d->h_out_ids + (size_t)buf * d->S;
    d->last_nseq = nseq;
    d->last_slots.assign(slots, slots + nseq);
    d->last_ids.assign(ids, ids + nseq);
    d->last_params.assign(d->h_params, d->h_params + nseq);
    if (out_ids) std::memcpy(out_ids, ids, nseq * 4);
    return LAIC_OK;
}

int laic_dev_reset_slot(laic_dev* d, int32_t slot) {
    if (!d || slot < 0 || slot >= d->S) return fail(LAIC_E_INVALID, "slot out of range");
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    CK(cudaStreamSynchronize(d->st));
    CK(cudaMemset(d->pos + slot, 0, 4));
    CK(cudaMemset(d->counts + (size_t)slot * d->V, 0, (size_t)d->V * 4));
    d->h_pos[slot] = 0;
    return LAIC_OK;
}

int laic_dev_slot_pos(laic_dev* d, int32_t slot, int64_t* pos) {
    if (!d || !pos || slot < 0 || slot >= d->S) return fail(LAIC_E_INVALID, "slot out of range");
    *pos = d->h_pos[slot];
    return LAIC_OK;
}

int laic_dev_fill_kv(laic_dev* d, int32_t slot, int32_t npos, uint64_t seed) {
    if (!d || slot < 0 || slot >= d->S) return fail(LAIC_E_INVALID, "slot out of range");
    if (npos < 0 || npos > d->cap) return fail(LAIC_E_CONTEXT, "context length exceeded");
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    if (npos > 0) {
        const long long slot_off = (long long)slot * d->kv_slot_stride;
        if (d->kv32)
            laic::fill_kv_kernel<float><<<1184, 256, 0, d->st>>>((float*)d->kc, (float*)d->vc, d->kv_layer_stride, slot_off,
                                                               d->Hkv, d->cap, d->D, npos, d->L, seed);
        else
            laic::fill_kv_kernel<__half><<<1184, 256, 0, d->st>>>((__half*)d->kc, (__half*)d->vc, d->kv_layer_stride,
                                                                slot_off, d->Hkv, d->cap, d->D, npos, d->L, seed);
        CK(cudaGetLastError());
    }
    CK(cudaMemcpyAsync(d->pos + slot, &npos, 4, cudaMemcpyHostToDevice, d->st));
    CK(cudaStreamSynchronize(d->st));
    d->h_pos[slot] = npos;
    return LAIC_OK;
}

int laic_dev_sync(laic_dev* d) {
    if (!d) return fail(LAIC_E_INVALID, "null device");
    CK(cudaSetDevice(d->device));
    CK(cudaStreamSynchronize(d->st));
    return LAIC_OK;
}

void* laic_dev_stream(laic_dev* d) { return d ? (void*)d->st : nullptr; }

int laic_dev_stats_get(laic_dev* d, laic_dev_stats* s) {
    if (!d || !s) return fail(LAIC_E_INVALID, "null argument");
    std::memset(s, 0, sizeof *s);
    uint64_t wb = 0;
    for (auto& l : d->layers) wb += l.qkv.bytes() + l.o.bytes() + l.gu.bytes() + l.down.bytes() + 8ull * d->h;
    wb += d->lm_head().bytes() + 4ull * d->h;
    s->weight_bytes = wb;
    s->kv_bytes_per_pos = (uint64_t)d->L * d->kv * 2 * (d->kv32 ? 4 : 2);
    s->launches_per_step = d->launches_step;  // of the most recently enqueued step (chained: + id record)
    s->launches_per_prefill = d->launches_prefill;
    s->attn_splits = d->last_split;
    s->tp_size = d->tp;
    return LAIC_OK;
}

int laic_dev_decode(laic_dev* d, int32_t nseq, const uint32_t* tokens, const int32_t* slots,
                    const laic_sample_params* params, int32_t nparams, int32_t steps, uint32_t* out_ids,
                    double* device_ms) {
    if (!d) return fail(LAIC_E_INVALID, "null device");
    if (steps < 1 || !out_ids) return fail(LAIC_E_INVALID, "steps must be >= 1 and out_ids non-null");
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    int rc = fill_inputs(d, nseq, tokens, slots);
    if (rc) return rc;
    for (int i = 0; i < nseq; ++i)
        if (d->h_pos[slots[i]] + steps > d->cap) return fail(LAIC_E_CONTEXT, "context length exceeded");
    if ((rc = fill_params(d, nseq, params, nparams))) return rc;
    const size_t need = (size_t)steps * nseq;
    if (need > d->hist_cap) {
        if (d->d_hist) cudaFree(d->d_hist);
        d->d_hist = nullptr;
        d->hist_cap = 0;
        CK(cudaMalloc(&d->d_hist, need * sizeof(unsigned)));
        d->hist_cap = need;
        for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);  // they captured the old buffer
        d->graphs.clear();
    }
    CK(cudaMemcpyAsync(d->d_tokens, d->h_tokens, nseq * 4, cudaMemcpyHostToDevice, d->st));
    CK(cudaMemcpyAsync(d->d_slots, d->h_slots, nseq * 4, cudaMemcpyHostToDevice, d->st));
    CK(cudaMemcpyAsync(d->d_params, d->h_params, nseq * sizeof(laic::SampleDev), cudaMemcpyHostToDevice, d->st));
    CK(cudaMemsetAsync(d->d_hist_count, 0, 4, d->st));
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0, d->st));
    for (int k = 0; k < steps && rc == LAIC_OK; ++k) rc = d->run(nseq, MODE_CHAIN);
    CK(cudaEventRecord(e1, d->st));
    CK(cudaStreamSynchronize(d->st));
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc) return rc;
    for (int i = 0; i < nseq; ++i) d->h_pos[slots[i]] += steps;
    if (device_ms) *device_ms = ms;
    CK(cudaMemcpy(out_ids, d->d_hist, need * sizeof(unsigned), cudaMemcpyDeviceToHost));
    return check_sampler_err(d);
}

int laic_dev_profile(laic_dev* d, int32_t nseq, const uint32_t* tokens, int32_t steps, laic_kernel_record* out,
                     int32_t max_out, int32_t* n_out) {
    if (!d || !tokens || steps < 1 || !out || !n_out) return fail(LAIC_E_INVALID, "bad argument");
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    std::vector<int32_t> slots(nseq);
    for (int i = 0; i < nseq; ++i) slots[i] = i;
    std::vector<laic_kernel_record> recs;
    int rc0 = d->reserve_scratch(nseq);
    if (rc0) return rc0;
    for (int it = 0; it < steps; ++it) {
        int rc = fill_inputs(d, nseq, tokens + (size_t)it * nseq, slots.data());
        if (rc) return rc;
        if ((rc = fill_params(d, nseq, nullptr, 0))) return rc;
        laic_dev::Timer t;
        // hold the stream while the host queues the step, so the events time the kernels, not the host
        laic::hold_kernel<<<1, 1, 0, d->st>>>(20000000LL);
        CK(cudaGetLastError());
        rc = d->enqueue(nseq, MODE_STEP, d->st, &t);
        CK(cudaStreamSynchronize(d->st));
        for (int i = 0; i < nseq; ++i) d->h_pos[i] += 1;
        for (size_t k = 0; k < t.ev.size(); ++k) {
            float ms = 0;
            cudaEventElapsedTime(&ms, t.ev[k].second.first, t.ev[k].second.second);
            cudaEventDestroy(t.ev[k].second.first);
            cudaEventDestroy(t.ev[k].second.second);
            auto it2 = std::find_if(recs.begin(), recs.end(),
                                    [&](const laic_kernel_record& r) { return t.ev[k].first == r.name; });
            if (it2 == recs.end()) {
                laic_kernel_record r{};
                std::snprintf(r.name, sizeof r.name, "%s", t.ev[k].first.c_str());
                recs.push_back(r);
                it2 = recs.end() - 1;
            }
            it2->launches += 1;
            it2->total_us += ms * 1000.0;
            it2->bytes += t.bytes[k];
        }
        if (rc) return rc;
    }
    *n_out = std::min<int32_t>(max_out, (int32_t)recs.size());
    for (int i = 0; i < *n_out; ++i) out[i] = recs[i];
    return LAIC_OK;
}

int laic_dev_step_trace(laic_dev* d, uint64_t* out, int64_t max_entries, int64_t* n, int32_t* ctas,
                        int32_t* phases) {
    if (!d || !out || !n || !ctas || !phases) return fail(LAIC_E_INVALID, "null argument");
    if (!d->ls_trace) return fail(LAIC_E_INVALID, "no step trace: create the engine with LAIC_FLAG_TRACE "
                                               "and run a one-sequence step on the persistent kernel");
    CK(cudaSetDevice(d->device));
    if (int rc_ = d->spec_cancel()) return rc_;  // (a pending speculative step assumed the old state)
    CK(cudaStreamSynchronize(d->st));
    const int64_t total = (int64_t)num_sms() * laic::ls_phases(d->L) * laic::ls_trace_stamps() +
                          (int64_t)num_sms() * laic::ls_trace_warp_words();
    *n = std::min(total, max_entries);
    *ctas = num_sms();
    *phases = laic::ls_phases(d->L);
    CK(cudaMemcpy(out, d->ls_trace, (size_t)*n * 8, cudaMemcpyDeviceToHost));
    return LAIC_OK;
}

int laic_blocks_convert(int32_t ggml_type, const void* src, uint64_t n, uint32_t flags, int32_t* out_type, void* dst,
                        uint64_t dst_cap, uint64_t* dst_bytes) {
    if (!src || !out_type || !dst_bytes) return fail(LAIC_E_INVALID, "null argument");
    if (n % 32) return fail(LAIC_E_INVALID, "element count must be a multiple of 32");
    const size_t in_bytes = elem_bytes(ggml_type, n);
    if (ggml_type != T_F32 && ggml_type != T_F16 && !in_bytes)
        return fail(LAIC_E_UNSUPPORTED, "unsupported GGML type " + std::to_string(ggml_type));
    std::vector<uint8_t> conv;
    int t = ggml_type;
    const bool c = convert_blocks(ggml_type, (const uint8_t*)src, n / 32, (flags & LAIC_FLAG_Q4_0_UPSTREAM) != 0, &t,
                                  conv);
    const size_t bytes = c ? conv.size() : in_bytes;
    *out_type = t;
    *dst_bytes = bytes;
    if (!dst) return LAIC_OK;  // size query
    if (dst_cap < bytes) return fail(LAIC_E_INVALID, "destination too small");
    std::memcpy(dst, c ? (const void*)conv.data() : src, bytes);
    return LAIC_OK;
}

int laic_nccl_unique_id(void* out128) {
    if (!out128) return fail(LAIC_E_INVALID, "null argument");
    std::string why;
    const laic::NcclApi* api = laic::nccl_api(why);
    if (!api) return fail(LAIC_E_NCCL, why);
    laic::ncclUniqueId id;
    const laic::ncclResult_t r = api->GetUniqueId(&id);
    if (r != laic::ncclSuccess) return fail(LAIC_E_NCCL, std::string("ncclGetUniqueId: ") + api->GetErrorString(r));
    std::memcpy(out128, &id, sizeof id);
    return LAIC_OK;
}

// ---- single tensors --------------------------------------------------------
}  // extern "C"

struct laic_tensor {
    int device = 0;
    Mat m;
    MvScratch sc;
};

extern "C" {

int laic_tensor_create(int32_t device, int32_t type, uint64_t in, uint64_t out, const void* data, size_t nbytes,
                       laic_tensor** t) {
    if (!data || !t || !in || !out) return fail(LAIC_E_INVALID, "bad argument");
    if (nbytes < elem_bytes(type, in * out)) return fail(LAIC_E_INVALID, "tensor data out of range");
    std::vector<uint8_t> conv;
    int ctype = type;
    if (convert_blocks(type, (const uint8_t*)data, in * out / 32, false, &ctype, conv)) {
        type = ctype;
        data = conv.data();
        nbytes = conv.size();
    }
    CK(cudaSetDevice(device));
    CK(laic::mv_set_attributes());
    std::unique_ptr<laic_tensor> x(new laic_tensor());
    x->device = device;
    int rc = mat_alloc(x->m, type, (int)out, (int)in);
    if (rc) return rc;
    cudaStream_t st;
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    rc = mat_fill(x->m, (const uint8_t*)data, (int)out, 1, 0, st);
    cudaStreamDestroy(st);
    if (rc) { mat_free(x->m); return rc; }
    *t = x.release();
    return LAIC_OK;
}

void laic_tensor_destroy(laic_tensor* t) {
    if (!t) return;
    cudaSetDevice(t->device);
    mat_free(t->m);
    mv_scratch_free(t->sc);
    delete t;
}

uint64_t laic_tensor_bytes(laic_tensor* t) { return t ? t->m.bytes() : 0; }

int laic_tensor_matvec(laic_tensor* t, const float* x, float* y, int32_t batch, void* stream) {
    if (!t || !x || !y || batch < 1) return fail(LAIC_E_INVALID, "bad argument");
    CK(cudaSetDevice(t->device));
    if (batch > 64) return fail(LAIC_E_UNSUPPORTED, "at most 64 sequences per matvec");
    const MvNeed need = mv_need(t->m, batch);
    int rc = mv_scratch_reserve(t->sc, need);
    if (rc) return rc;
    // split-K tickets start at zero: a launch whose wait ran out may have left some raised
    if (need.ntiles) CK(cudaMemsetAsync(t->sc.tile_cnt, 0, need.ntiles * 4, (cudaStream_t)stream));
    laic::MvParams p{};
    p.nseq = batch; p.x = x; p.ldx = t->m.in; p.out = y; p.ldo = t->m.rows;
    CK(launch_matvec(t->m, p, laic::EPI_STORE, false, t->sc, (cudaStream_t)stream, false));
    return LAIC_OK;
}

int laic_tensor_dequant(laic_tensor* t, float* out, void* stream) {
    if (!t || !out) return fail(LAIC_E_INVALID, "bad argument");
    CK(cudaSetDevice(t->device));
    laic::tile_dequant_kernel<<<1184, 256, 0, (cudaStream_t)stream>>>(t->m.type, t->m.q, t->m.s, t->m.in, t->m.nb,
                                                                       t->m.rows, out);
    CK(cudaGetLastError());
    return LAIC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// laic_tensor_matvec_noalloc: the single-tensor product with fixed working memory
// ---------------------------------------------------------------------------
// Some hosts hand all device memory to their own arena at start-up (weights,
// KV cache) and must not call the CUDA allocator afterwards: cudaMalloc and
// cudaFree may synchronise the device and stall every stream, and a failed
// allocation in the middle of a request cannot be recovered there. For them
// the entry point below takes its working memory (split-K partials and
// tickets, prepared activations, error flag) from one array compiled into
// this library instead of from the allocator.
//
// The array is shared by every call on a device and keeps whatever the last
// call left in it; the ticket counters, which must start at zero, are cleared
// on the stream at the start of every call. The error word at its start is
// sticky: a bounded wait that runs out sets it, and only laic_tensor_check
// reads and clears it. Two calls whose kernels overlap in time (different
// streams, or host threads without ordering) race on the array.
namespace {

constexpr size_t kFixedScratchBytes = LAIC_FIXED_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_fixed_scratch[kFixedScratchBytes];

constexpr int kFixedMaxDevices = 64;
std::mutex g_fixed_mu;
unsigned char* g_fixed_base[kFixedMaxDevices] = {};

// Device address of the array on `device` (which must be current); looked up
// once per device, at that device's first call, and kept for the life of the
// process (a cudaDeviceReset would invalidate it: the library does not support
// being used across one).
int fixed_scratch_base(int device, unsigned char** base) {
    if (device < 0 || device >= kFixedMaxDevices) return fail(LAIC_E_INVALID, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_fixed_mu);
    if (!g_fixed_base[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_fixed_scratch);
        if (e != cudaSuccess) return fail(LAIC_E_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_fixed_base[device] = static_cast<unsigned char*>(p);
    }
    *base = g_fixed_base[device];
    return LAIC_OK;
}

size_t round256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace

extern "C" {

int laic_tensor_matvec_noalloc(laic_tensor* t, const float* x, float* y, int32_t batch, void* stream) {
    if (!t || !x || !y || batch < 1) return fail(LAIC_E_INVALID, "bad argument");
    CK(cudaSetDevice(t->device));
    if (batch > 64) return fail(LAIC_E_UNSUPPORTED, "at most 64 sequences per matvec");
    const MvNeed need = mv_need(t->m, batch);
    // carve: [error word (sticky)] [tickets (cleared each call)] [partials] [activations] [split scales]
    const size_t zero_bytes = round256(need.ntiles * 4);
    const size_t part_off = 256 + zero_bytes;
    const size_t xg_off = part_off + round256(need.part_floats * 4);
    const size_t xinv_off = xg_off + round256(need.xg_bytes);
    const size_t total = xinv_off + round256(need.xinv_floats * 4);
    if (total > kFixedScratchBytes)
        return fail(LAIC_E_INVALID, "laic_tensor_matvec_noalloc: this matrix at batch " + std::to_string(batch) +
                                        " needs " + std::to_string(total) + " bytes of working memory, more than the " +
                                        std::to_string(kFixedScratchBytes) + " bytes of the fixed array");
    unsigned char* base = nullptr;
    int rc = fixed_scratch_base(t->device, &base);
    if (rc) return rc;
    const cudaStream_t st = (cudaStream_t)stream;
    if (zero_bytes) CK(cudaMemsetAsync(base + 256, 0, zero_bytes, st));
    MvScratch sc;
    sc.err = reinterpret_cast<int*>(base);
    sc.tile_cnt = reinterpret_cast<unsigned*>(base + 256);
    sc.part = reinterpret_cast<float*>(base + part_off);
    sc.xg = base + xg_off;
    sc.xinv = reinterpret_cast<float*>(base + xinv_off);
    laic::MvParams p{};
    p.nseq = batch; p.x = x; p.ldx = t->m.in; p.out = y; p.ldo = t->m.rows;
    CK(launch_matvec(t->m, p, laic::EPI_STORE, false, sc, st, false));
    return LAIC_OK;
}

int laic_tensor_check(laic_tensor* t, void* stream) {
    if (!t) return fail(LAIC_E_INVALID, "bad argument");
    CK(cudaSetDevice(t->device));
    const cudaStream_t st = (cudaStream_t)stream;
    CK(cudaStreamSynchronize(st));
    int own = 0, fixed = 0;
    if (t->sc.err) CK(cudaMemcpy(&own, t->sc.err, 4, cudaMemcpyDeviceToHost));
    unsigned char* base = nullptr;
    if (int rc = fixed_scratch_base(t->device, &base)) return rc;
    CK(cudaMemcpy(&fixed, base, 4, cudaMemcpyDeviceToHost));
    if (own) CK(cudaMemset(t->sc.err, 0, 4));
    if (fixed) CK(cudaMemset(base, 0, 4));
    if (own || fixed) return fail(LAIC_E_CUDA, wait_error_text(own ? own : fixed));
    return LAIC_OK;
}

int laic_selftest_peer_timeout(int32_t device, int64_t spin_cycles, int32_t* code) {
    if (!code || spin_cycles <= 0) return fail(LAIC_E_INVALID, "bad argument");
    *code = 0;
    CK(cudaSetDevice(device));
    // rank 0 of two; "rank 1" is a mailbox on this GPU that nothing ever writes
    const int n = 1024;
    const size_t box_floats = (size_t)2 * 2 * n, flag_words = (size_t)2 * 2 * laic::kArCtas;
    float *x = nullptr, *box0 = nullptr, *box1 = nullptr;
    unsigned *fl0 = nullptr, *fl1 = nullptr, *ctr = nullptr;
    int* err = nullptr;
    auto release = [&]() {
        for (void* b : {(void*)x, (void*)box0, (void*)box1, (void*)fl0, (void*)fl1, (void*)ctr, (void*)err})
            if (b) cudaFree(b);
    };
    cudaError_t e = cudaSuccess;
    for (auto [ptr, bytes] : {std::pair<void**, size_t>{(void**)&x, n * 4}, {(void**)&box0, box_floats * 4},
                              {(void**)&box1, box_floats * 4}, {(void**)&fl0, flag_words * 4},
                              {(void**)&fl1, flag_words * 4}, {(void**)&ctr, 8}, {(void**)&err, 4}}) {
        if (e == cudaSuccess) e = cudaMalloc(ptr, bytes);
        if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    }
    if (e == cudaSuccess) {
        laic::ArParams ap{};
        ap.x = x; ap.n = n; ap.rank = 0; ap.ranks = 2; ap.nmax = n;
        ap.box[0] = box0; ap.box[1] = box1; ap.flags[0] = fl0; ap.flags[1] = fl1;
        ap.epoch = ctr; ap.done = ctr + 1; ap.err = err; ap.spin_limit = spin_cycles;
        laic::allreduce_oneshot_kernel<<<laic::kArCtas, laic::kArThreads>>>(ap);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(code, err, 4, cudaMemcpyDeviceToHost);
    }
    release();
    if (e != cudaSuccess) return fail(LAIC_E_CUDA, std::string("self-test: ") + cudaGetErrorString(e));
    if (*code) return fail(LAIC_E_CUDA, wait_error_text(*code));
    return LAIC_OK;
}

}  // extern "C"
