// Split-K GQA decode attention over the device KV cache.
//
// Replaces the attention lambda of LlamaRuntime::step (reference
// src/inference_v2.cpp:31): per query head h (kv head kh = h / (H/Hkv)),
// s_t = (q_h . k_t) / sqrt(d), softmax over t <= pos, out = sum_t p_t v_t.
//
// Grid (split, kv_head, seq); one CTA walks a contiguous run of 32-position
// tiles of one (sequence, kv head) pair for all H/Hkv query heads of its
// group, so every K and V row is read from HBM once per step. Inside a tile,
// lane = position for the scores (q broadcast from shared memory) and
// lane = head dimension for the V accumulation, with an online softmax per
// warp. The CTA's partial (max, sum, unnormalised output) goes to a scratch
// buffer; the last CTA of the pair (atomic ticket, no spinning) merges the
// splits with the usual log-sum-exp weights and writes the output.
//
// KV cache layout: [slot][kv_head][position][head_dim] per layer, FP16 (or
// FP32 in the parity mode, where scores use the reference's unfused
// sequential multiply-add order).
#pragma once
#include "common.cuh"

namespace laic {

struct AttnParams {
    const float* q;            // [nseq][ldq], heads contiguous
    int ldq;
    float* out;                // [nseq][ldo]
    int ldo;
    const void* kc;            // this layer's K cache
    const void* vc;            // this layer's V cache
    long long slot_stride;     // elements between slots
    int cap;                   // positions per slot
    int heads, kv_heads;
    const int* slots;          // [nseq]
    const int* pos;            // [max_seqs]; the sequence attends to positions 0..pos
    int nsplit;
    float* part;               // [nseq][kv_heads][nsplit][G][D+2] (scratch)
    unsigned* counters;        // [nseq][kv_heads], zero between launches (scratch)
    float sqrt_d;
};

template <typename KV, int N> struct KvLoad;
template <> struct KvLoad<__half, 1> {
    static __device__ __forceinline__ void load(const __half* p, float* o) { o[0] = __half2float(*p); }
};
template <> struct KvLoad<__half, 2> {
    static __device__ __forceinline__ void load(const __half* p, float* o) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p));
        o[0] = f.x; o[1] = f.y;
    }
};
template <> struct KvLoad<__half, 4> {
    static __device__ __forceinline__ void load(const __half* p, float* o) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
    }
};
template <> struct KvLoad<__half, 8> {
    static __device__ __forceinline__ void load(const __half* p, float* o) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            o[2 * i] = f.x; o[2 * i + 1] = f.y;
        }
    }
};
template <int N> struct KvLoad<float, N> {
    static __device__ __forceinline__ void load(const float* p, float* o) {
        if constexpr (N % 4 == 0) {
#pragma unroll
            for (int i = 0; i < N; i += 4) {
                const float4 f = *reinterpret_cast<const float4*>(p + i);
                o[i] = f.x; o[i + 1] = f.y; o[i + 2] = f.z; o[i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i) o[i] = p[i];
        }
    }
};

constexpr int kAttnWarps = 4;

template <int D, int GMAX, typename KV, bool EXACT>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(const AttnParams p) {
    constexpr int DPL = D / 32 > 0 ? D / 32 : 1;  // head dims per lane in the V phase
    constexpr int NW = kAttnWarps;
    __shared__ float qs[GMAX][D];
    __shared__ float ps[NW][GMAX][32];
    __shared__ float cm[NW][GMAX], cl[NW][GMAX];
    __shared__ float cacc[NW][GMAX][D];
    __shared__ int is_last;

    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = p.heads / p.kv_heads;

    pdl_wait();
    const int slot = p.slots[seq];
    const int n = p.pos[slot] + 1;
    const int ntiles = (n + 31) >> 5;
    const int tps = (ntiles + p.nsplit - 1) / p.nsplit;
    const int tile0 = split * tps, tile1 = min(ntiles, tile0 + tps);
    const int t1 = min(n, tile1 * 32);

    for (int i = threadIdx.x; i < G * D; i += blockDim.x)
        qs[i / D][i % D] = p.q[(size_t)seq * p.ldq + (size_t)kvh * G * D + i];
    __syncthreads();
    pdl_launch_dependents();

    const KV* kb = reinterpret_cast<const KV*>(p.kc) + (size_t)slot * p.slot_stride + (size_t)kvh * p.cap * D;
    const KV* vb = reinterpret_cast<const KV*>(p.vc) + (size_t)slot * p.slot_stride + (size_t)kvh * p.cap * D;

    float m[GMAX], l[GMAX], acc[GMAX][DPL];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
        m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
        for (int k = 0; k < DPL; ++k) acc[g][k] = 0.f;
    }

    for (int tile = tile0 + warp; tile < tile1; tile += NW) {
        const int base = tile * 32, t = base + lane;
        const bool valid = t < t1;
        float s[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g) s[g] = 0.f;
        if (valid) {
            const KV* kr = kb + (size_t)t * D;
            // the whole key row first (all loads in flight), then the dot products
            float kf[D];
#pragma unroll
            for (int ch = 0; ch < D; ch += 8) KvLoad<KV, 8>::load(kr + ch, kf + ch);
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                if (g < G) {
#pragma unroll
                    for (int d = 0; d < D; ++d) {
                        if (EXACT) s[g] = __fadd_rn(s[g], __fmul_rn(qs[g][d], kf[d]));
                        else s[g] = fmaf(qs[g][d], kf[d], s[g]);
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < GMAX; ++g) s[g] = s[g] / p.sqrt_d;
        } else {
#pragma unroll
            for (int g = 0; g < GMAX; ++g) s[g] = -INFINITY;
        }
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            if (g < G) {
                const float mnew = fmaxf(m[g], warp_max(s[g]));
                const float corr = expf(m[g] - mnew);
                const float pv = valid ? expf(s[g] - mnew) : 0.f;
                l[g] = l[g] * corr + warp_sum(pv);
                m[g] = mnew;
#pragma unroll
                for (int k = 0; k < DPL; ++k) acc[g][k] *= corr;
                ps[warp][g][lane] = pv;
            }
        }
        __syncwarp();
        const int cnt = min(32, t1 - base);
        const KV* vrow = vb + (size_t)base * D + lane * DPL;
        int j = 0;
        for (; j + 8 <= cnt; j += 8) {  // eight value rows in flight
            float vf[8][DPL];
#pragma unroll
            for (int u = 0; u < 8; ++u) KvLoad<KV, DPL>::load(vrow + (size_t)(j + u) * D, vf[u]);
#pragma unroll
            for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int g = 0; g < GMAX; ++g) {
                    if (g < G) {
                        const float pj = ps[warp][g][j + u];
#pragma unroll
                        for (int k = 0; k < DPL; ++k) acc[g][k] = fmaf(pj, vf[u][k], acc[g][k]);
                    }
                }
        }
        for (; j < cnt; ++j) {
            float vf[DPL];
            KvLoad<KV, DPL>::load(vrow + (size_t)j * D, vf);
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                if (g < G) {
                    const float pj = ps[warp][g][j];
#pragma unroll
                    for (int k = 0; k < DPL; ++k) acc[g][k] = fmaf(pj, vf[k], acc[g][k]);
                }
            }
        }
        __syncwarp();
    }

    // ---- merge the warps of this CTA
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
        if (g < G) {
            if (lane == 0) { cm[warp][g] = m[g]; cl[warp][g] = l[g]; }
#pragma unroll
            for (int k = 0; k < DPL; ++k)
                if (lane * DPL + k < D) cacc[warp][g][lane * DPL + k] = acc[g][k];
        }
    }
    __syncthreads();

    const size_t pair = (size_t)seq * p.kv_heads + kvh;
    const int PD = D + 2;
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, dd = i % D;
        float M = -INFINITY;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, cm[w][g]);
        float L = 0.f, A = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < NW; ++w) {
                const float e = expf(cm[w][g] - M);
                L = fmaf(cl[w][g], e, L);
                A = fmaf(cacc[w][g][dd], e, A);
            }
        }
        if (p.nsplit == 1) {
            p.out[(size_t)seq * p.ldo + ((size_t)kvh * G + g) * D + dd] = A / L;
        } else {
            float* dst = p.part + ((pair * p.nsplit + split) * G + g) * PD;
            dst[dd] = A;
            if (dd == 0) { dst[D] = M; dst[D + 1] = L; }
        }
    }
    if (p.nsplit == 1) return;

    // ---- last CTA of this (seq, kv head) merges the splits
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned ticket = atomicAdd(p.counters + pair, 1u);
        is_last = ticket == (unsigned)(p.nsplit - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, dd = i % D;
        const float* src = p.part + (pair * p.nsplit * G + g) * PD;
        const size_t sstride = (size_t)G * PD;
        float M = -INFINITY;
        for (int j = 0; j < p.nsplit; ++j) M = fmaxf(M, __ldcg(src + j * sstride + D));
        float L = 0.f, A = 0.f;
        for (int j = 0; j < p.nsplit; ++j) {
            const float mj = __ldcg(src + j * sstride + D);
            if (mj == -INFINITY) continue;
            const float e = expf(mj - M);
            L = fmaf(__ldcg(src + j * sstride + D + 1), e, L);
            A = fmaf(__ldcg(src + j * sstride + dd), e, A);
        }
        p.out[(size_t)seq * p.ldo + ((size_t)kvh * G + g) * D + dd] = A / L;
    }
    if (threadIdx.x == 0) p.counters[pair] = 0u;
}

}  // namespace laic
