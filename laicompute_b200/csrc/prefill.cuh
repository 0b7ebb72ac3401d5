// Batched prompt prefill: the prompt's tokens of one sequence go through every
// layer together, with the projections as dense fp16 tensor-core GEMMs
// (gemm_sm100.cu), instead of one LlamaRuntime::step per token (reference
// src/inference_v2.cpp:34 feeds the prompt through step() one token at a
// time). The elementwise work between the GEMMs is here; attention reuses the
// decode attention kernel with one causal length per query row.
//
// Precision: weights are dequantised to binary16 (q * d rounded, 2^-12
// relative) and the GEMM inputs are binary16; accumulation is FP32. The KV
// cache this writes is FP16 in any case.
#pragma once
#include "common.cuh"
#include "tiles.cuh"

namespace laic {

// out[r][i] = binary16 of the decoded weight (fragment-tile layout in, row-major out).
__global__ void dequant_f16_kernel(int type, const uint8_t* q, const uint8_t* s, int nb, int rows, __half* out) {
    const int in = nb * 32;
    const size_t n = (size_t)rows * in;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / in), i = (int)(e - (size_t)r * in);
        out[e] = __float2half_rn(tile_value(type, q, s, nb, r, i));
    }
}

// One row per CTA: A[t][:] = binary16(x * (inv * w)), inv = 1/sqrt(mean(x^2) + eps) (w null: no norm).
__global__ void rmsnorm_f16_kernel(const float* x, int ldx, const float* w, float eps, int n, __half* a, int lda) {
    __shared__ float red[32];
    const float* xr = x + (size_t)blockIdx.x * ldx;
    __half* ar = a + (size_t)blockIdx.x * lda;
    float inv = 1.f;
    if (w) {
        float ss = 0.f;
        for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
        ss = block_sum(ss, red);
        inv = 1.f / sqrtf(ss / float(n) + eps);
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) ar[i] = __float2half_rn(w ? xr[i] * (inv * w[i]) : xr[i]);
}

// QKV rows of every token: RoPE (adjacent pairs) on q and k at position p0 + t, q out in FP32,
// K and V appended to the slot's FP16 cache.
struct QkvPostParams {
    const float* c;        // [T][hq + 2 kv]
    int T, hq, kv, head_dim, rope_pairs, p0;
    const float2* rope_cs; // [ctx][rope_pairs]
    float* q;              // [T][hq]
    __half* kc;            // this layer's K cache, the slot's base
    __half* vc;
    int cap;
};
__global__ void qkv_post_kernel(const QkvPostParams p) {
    const int w = p.hq + 2 * p.kv;
    const size_t n = (size_t)p.T * w;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(e / w), r = (int)(e - (size_t)t * w);
        const float v = p.c[e];
        int rr = r, region = 0;
        if (rr >= p.hq) { rr -= p.hq; region = 1; if (rr >= p.kv) { rr -= p.kv; region = 2; } }
        const int d = rr % p.head_dim, ps = p.p0 + t;
        float o = v;
        if (region < 2 && d < 2 * p.rope_pairs) {
            const float other = p.c[e ^ 1];  // the pair partner (rows 2i, 2i+1; row widths are even)
            const float2 cs = p.rope_cs[(size_t)ps * p.rope_pairs + (d >> 1)];
            if ((d & 1) == 0) o = __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(other, cs.y));
            else o = __fadd_rn(__fmul_rn(other, cs.y), __fmul_rn(v, cs.x));
        }
        if (region == 0) {
            p.q[(size_t)t * p.hq + rr] = o;
        } else {
            __half* base = region == 1 ? p.kc : p.vc;
            base[((size_t)(rr / p.head_dim) * p.cap + ps) * p.head_dim + d] = __float2half_rn(o);
        }
    }
}

// x += c (the residual add of o and down), n elements.
__global__ void residual_add_kernel(float* x, const float* c, size_t n) {
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        x[e] += c[e];
}

// act[t][o] = binary16(silu(gate) * up), gate/up rows interleaved in c[t][2o], c[t][2o+1].
__global__ void swiglu_f16_kernel(const float* c, int T, int F, __half* act) {
    const size_t n = (size_t)T * F;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(e / F), o = (int)(e - (size_t)t * F);
        const float g = c[(size_t)t * 2 * F + 2 * o], u = c[(size_t)t * 2 * F + 2 * o + 1];
        act[e] = __float2half_rn((g / (1.f + expf(-g))) * u);
    }
}

__global__ void to_f16_kernel(const float* src, __half* dst, size_t n) {
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        dst[e] = __float2half_rn(src[e]);
}

// The prefilled slot moves past its prompt; per-row slots and positions for the attention.
__global__ void prefill_rows_kernel(int slot, int p0, int T, int* slots, int* npos) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
        slots[t] = slot;
        npos[t] = p0 + t;
    }
}
__global__ void add_pos_kernel(int* pos, int slot, int n) {
    if (threadIdx.x == 0 && blockIdx.x == 0) pos[slot] += n;
}

}  // namespace laic
