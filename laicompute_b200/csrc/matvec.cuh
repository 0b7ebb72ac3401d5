// Dequant-fused matrix-vector product for decode (CUDA cores, FP32 accumulate).
//
// Replaces LlamaRuntime::matvec (reference src/inference_v2.cpp:29) with its
// two row-dot paths quant_dot (:21, quant_v2::value per element) and
// dot_cached (:22, compute::dot_f16). Each projection of a layer is one
// launch that also carries the elementwise work around it:
//   prologue  rmsnorm of the residual (src/inference_v2.cpp:24, LlamaRuntime::norm :30)
//   epilogue  store | residual add (compute::axpy_f32, src/compute_dot.cpp:64-72)
//             | SwiGLU (gate/up rows interleaved, :23 and :31)
//             | QKV: RoPE (:25) on q and k, then K/V appended to the device cache
//
// Device weight layout (built once at upload from the GGUF blocks, bytes unchanged):
//   Q4_0  qs plane: 16 B per block [rows][nb] (the block's nibble bytes)
//         d  plane: binary16 per block [rows][nb]
//   Q8_0  qs plane: 32 B per block [rows][nb] (the block's int8 quants)
//         d  plane: binary16 per block [rows][nb]
//   F16   [rows][in] binary16, as in the file
// so every 16-byte load is aligned and a warp reads 512 contiguous bytes of a row.
//
// Work split: a warp owns RG consecutive rows; lane l handles the 32-element
// blocks c = l, l+32, ... of those rows, keeping that block's activations in
// registers for all RG rows. Per-row partial sums are reduced across the warp
// with a transposed butterfly (one shuffle per row per lane).
//
// Q4_0 decode: a nibble n at bit 4k of a 32-bit word becomes the float
// 2^23 + n*2^(4k) with one AND|OR (exponent 0x4B), and (n-8)*2^(4k) after one
// subtraction; the activation it multiplies was pre-scaled by 2^-4k in shared
// memory, so every product is exact before accumulation. Q8_0 uses a byte
// permute into the same exponent field. The block scale d is applied once
// per block: y += d * sum_i (q_i - 8) x_i.
#pragma once
#include "common.cuh"

namespace laic {

enum : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

struct MatvecParams {
    const void* w;             // qs plane (Q4_0/Q8_0) or rows (F16)
    const unsigned short* d;   // scale plane (Q4_0/Q8_0)
    int rows, in, nb;          // nb = in / 32
    int nseq;
    const float* x;            // input [nseq][ldx]
    int ldx;
    const float* norm_w;       // rmsnorm weight [in] (nullptr: no norm)
    float eps;
    float* out;                // epilogue output
    int ldo;
    // EPI_QKV
    int q_rows, kv_rows, head_dim, rope_pairs;
    const float2* rope_cs;     // [ctx][rope_pairs] (cos, sin)
    const int* slots;          // [nseq] slot of each sequence
    const int* pos;            // [max_seqs] position of each slot
    void* kc;                  // this layer's K cache base
    void* vc;                  // this layer's V cache base
    long long kv_slot_stride;  // elements between slots
    int kv_cap;                // positions per slot
};

template <int WT> struct WT_ {
};
template <> struct WT_<T_Q4_0> { static constexpr int VEC = 1, RG = 8; };
template <> struct WT_<T_Q8_0> { static constexpr int VEC = 2, RG = 8; };
template <> struct WT_<T_F16> { static constexpr int VEC = 4, RG = 4; };

// x layout in shared memory: block c of 32 floats holds its eight 16-byte
// chunks in XOR-swizzled order (chunk q at q ^ (c & 7)) so the eight lanes
// reading eight consecutive blocks hit distinct banks.
__device__ __forceinline__ int xs_index(int e) {
    const int c = e >> 5, q = (e >> 2) & 7;
    return (c << 5) | ((q ^ (c & 7)) << 2) | (e & 3);
}

// Power-of-two pre-scale of activation e for the Q4_0 exponent trick.
__device__ __forceinline__ float q4_prescale(int e) {
    const int k = e & 7;
    const int sh = 4 * (k < 5 ? k : k - 3);
    return __int_as_float((127 - sh) << 23);
}

template <int NS>
__device__ __forceinline__ void dot_q4_0(const uint4 q, const float (&x)[NS][32], float (&r)[NS]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    const float M = 8388608.f;
#pragma unroll
    for (int s = 0; s < NS; ++s) r[s] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t a = w[i], u = a >> 12;
        float f[8];
        f[0] = __int_as_float((a & 0x0000000Fu) | 0x4B000000u) - (M + 8.f);
        f[1] = __int_as_float((a & 0x000000F0u) | 0x4B000000u) - (M + 128.f);
        f[2] = __int_as_float((a & 0x00000F00u) | 0x4B000000u) - (M + 2048.f);
        f[3] = __int_as_float((a & 0x0000F000u) | 0x4B000000u) - (M + 32768.f);
        f[4] = __int_as_float((a & 0x000F0000u) | 0x4B000000u) - (M + 524288.f);
        f[5] = __int_as_float((u & 0x00000F00u) | 0x4B000000u) - (M + 2048.f);
        f[6] = __int_as_float((u & 0x0000F000u) | 0x4B000000u) - (M + 32768.f);
        f[7] = __int_as_float((u & 0x000F0000u) | 0x4B000000u) - (M + 524288.f);
#pragma unroll
        for (int s = 0; s < NS; ++s)
#pragma unroll
            for (int k = 0; k < 8; ++k) r[s] = fmaf(f[k], x[s][8 * i + k], r[s]);
    }
}

template <int NS>
__device__ __forceinline__ void dot_q8_0(const uint4 q0, const uint4 q1, const float (&x)[NS][32], float (&r)[NS]) {
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const float C = 8388608.f + 128.f;
#pragma unroll
    for (int s = 0; s < NS; ++s) r[s] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t u = w[i] ^ 0x80808080u;
        float f[4];
        f[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - C;
        f[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - C;
        f[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - C;
        f[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - C;
#pragma unroll
        for (int s = 0; s < NS; ++s)
#pragma unroll
            for (int k = 0; k < 4; ++k) r[s] = fmaf(f[k], x[s][4 * i + k], r[s]);
    }
}

template <int NS>
__device__ __forceinline__ void dot_f16(const uint4 (&q)[4], const float (&x)[NS][32], float (&r)[NS]) {
#pragma unroll
    for (int s = 0; s < NS; ++s) r[s] = 0.f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const uint32_t w[4] = {q[v].x, q[v].y, q[v].z, q[v].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
#pragma unroll
            for (int s = 0; s < NS; ++s) {
                r[s] = fmaf(f.x, x[s][8 * v + 2 * i], r[s]);
                r[s] = fmaf(f.y, x[s][8 * v + 2 * i + 1], r[s]);
            }
        }
    }
}

// Reduce V per-lane partials over the warp; lane l ends with value idx(l).
template <int V>
__device__ __forceinline__ float transpose_reduce(float (&v)[V], int lane, int& idx) {
    int cnt = V;
    idx = 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        if (cnt > 1) {
            const int half = cnt >> 1;
            const bool upper = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < half) {
                    const float send = upper ? v[i] : v[i + half];
                    const float keep = upper ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            if (upper) idx += half;
            cnt = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
        }
    }
    return v[0];
}

// Lane offset holding the value whose index differs by `w` (a power of two < V).
template <int V>
__host__ __device__ constexpr int partner_offset(int w) {
    int cnt = V, off = 16;
    while (cnt > 1) {
        if ((cnt >> 1) == w) return off;
        cnt >>= 1;
        off >>= 1;
    }
    return 0;
}
// Lanes holding the same value: the low log2(32/V) lane bits.
template <int V>
__host__ __device__ constexpr int dup_mask() {
    int cnt = V, off = 16;
    while (cnt > 1) { cnt >>= 1; off >>= 1; }
    return off == 0 ? 0 : off * 2 - 1;
}

template <typename KV> __device__ __forceinline__ KV to_kv(float v);
template <> __device__ __forceinline__ __half to_kv<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float to_kv<float>(float v) { return v; }

template <int WT, int NS, int EPI, typename KV>
__global__ void __launch_bounds__(256, NS == 1 ? 2 : 1) matvec_kernel(const MatvecParams p) {
    constexpr int VEC = WT_<WT>::VEC, RG = WT_<WT>::RG, V = RG * NS;
    extern __shared__ float xs[];  // [NS][in], swizzled
    __shared__ float red[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ngroups = (p.rows + RG - 1) / RG;

    pdl_wait();
    for (int s0 = 0; s0 < p.nseq; s0 += NS) {
        // ---- prologue: activations (optionally rmsnorm'd) into shared memory
        __syncthreads();
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            const int seq = s0 + s;
            float* dst = xs + s * p.in;
            if (seq >= p.nseq) {
                for (int e = threadIdx.x; e < p.in; e += blockDim.x) dst[e] = 0.f;
                continue;
            }
            const float* src = p.x + (size_t)seq * p.ldx;
            float inv = 1.f;
            if (p.norm_w) {
                float ss = 0.f;
                for (int e = threadIdx.x; e < p.in; e += blockDim.x) { const float v = src[e]; ss = fmaf(v, v, ss); }
                ss = block_sum(ss, red);
                inv = 1.f / sqrtf(ss / float(p.in) + p.eps);
            }
            for (int e = threadIdx.x; e < p.in; e += blockDim.x) {
                float v = src[e];
                if (p.norm_w) v = v * (inv * p.norm_w[e]);
                if (WT == T_Q4_0) v *= q4_prescale(e);
                dst[xs_index(e)] = v;
            }
        }
        __syncthreads();
        if (s0 + NS >= p.nseq) pdl_launch_dependents();

        // ---- row groups
        for (int g = blockIdx.x * 8 + warp; g < ngroups; g += gridDim.x * 8) {
            const int r0 = g * RG;
            float acc[RG * NS];
#pragma unroll
            for (int i = 0; i < RG * NS; ++i) acc[i] = 0.f;

            for (int c = lane; c < p.nb; c += 32) {
                float xr[NS][32];
#pragma unroll
                for (int s = 0; s < NS; ++s) {
                    const float4* xb = reinterpret_cast<const float4*>(xs + s * p.in + c * 32);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 t = xb[q ^ (c & 7)];
                        xr[s][4 * q] = t.x; xr[s][4 * q + 1] = t.y; xr[s][4 * q + 2] = t.z; xr[s][4 * q + 3] = t.w;
                    }
                }
                uint4 wq[RG][VEC];
                float dsc[RG];
#pragma unroll
                for (int r = 0; r < RG; ++r) {
                    const int row = r0 + r < p.rows ? r0 + r : p.rows - 1;
                    if (WT == T_F16) {
                        const uint4* src = reinterpret_cast<const uint4*>(
                            reinterpret_cast<const __half*>(p.w) + (size_t)row * p.in + c * 32);
#pragma unroll
                        for (int v = 0; v < VEC; ++v) wq[r][v] = ldg_stream(src + v);
                        dsc[r] = 1.f;
                    } else {
                        const uint4* src = reinterpret_cast<const uint4*>(p.w) + ((size_t)row * p.nb + c) * VEC;
#pragma unroll
                        for (int v = 0; v < VEC; ++v) wq[r][v] = ldg_stream(src + v);
                        dsc[r] = h2f_bits(ldg_u16(p.d + (size_t)row * p.nb + c));
                    }
                }
#pragma unroll
                for (int r = 0; r < RG; ++r) {
                    float part[NS];
                    if (WT == T_Q4_0) dot_q4_0<NS>(wq[r][0], xr, part);
                    else if (WT == T_Q8_0) dot_q8_0<NS>(wq[r][0], wq[r][VEC - 1], xr, part);
                    else {
                        uint4 t[4];
#pragma unroll
                        for (int v = 0; v < 4; ++v) t[v] = wq[r][v < VEC ? v : 0];
                        dot_f16<NS>(t, xr, part);
                    }
#pragma unroll
                    for (int s = 0; s < NS; ++s) acc[r * NS + s] = fmaf(dsc[r], part[s], acc[r * NS + s]);
                }
            }

            int idx;
            const float val = transpose_reduce<V>(acc, lane, idx);
            const int r = r0 + idx / NS, seq = s0 + idx % NS;
            constexpr int POFF = partner_offset<V>(NS);  // lane holding row r^1, same seq
            const float pval = __shfl_xor_sync(0xffffffffu, val, POFF);
            const bool writer = (lane & dup_mask<V>()) == 0 && r < p.rows && seq < p.nseq;

            if (EPI == EPI_STORE) {
                if (writer) p.out[(size_t)seq * p.ldo + r] = val;
            } else if (EPI == EPI_ADD) {
                if (writer) p.out[(size_t)seq * p.ldo + r] += val;
            } else if (EPI == EPI_SWIGLU) {
                // row 2o = gate o, row 2o+1 = up o: out[o] = silu(gate) * up
                if (writer && (r & 1) == 0) {
                    const float gte = val, up = pval;
                    p.out[(size_t)seq * p.ldo + (r >> 1)] = (gte / (1.f + expf(-gte))) * up;
                }
            } else {  // EPI_QKV
                if (writer) {
                    const int slot = p.slots[seq], ps = p.pos[slot];
                    int rr = r, region = 0;  // 0 q, 1 k, 2 v
                    if (rr >= p.q_rows) { rr -= p.q_rows; region = 1; if (rr >= p.kv_rows) { rr -= p.kv_rows; region = 2; } }
                    const int i = rr % p.head_dim;
                    float outv = val;
                    if (region < 2 && i < 2 * p.rope_pairs) {
                        const float2 cs = p.rope_cs[(size_t)ps * p.rope_pairs + (i >> 1)];
                        // adjacent-pair rotation, unfused to match the reference's rounding
                        if ((i & 1) == 0) outv = __fsub_rn(__fmul_rn(val, cs.x), __fmul_rn(pval, cs.y));
                        else outv = __fadd_rn(__fmul_rn(pval, cs.y), __fmul_rn(val, cs.x));
                    }
                    if (region == 0) {
                        p.out[(size_t)seq * p.ldo + rr] = outv;
                    } else {
                        const int kvh = rr / p.head_dim;
                        KV* base = reinterpret_cast<KV*>(region == 1 ? p.kc : p.vc);
                        base[(size_t)slot * p.kv_slot_stride + ((size_t)kvh * p.kv_cap + ps) * p.head_dim + i] =
                            to_kv<KV>(outv);
                    }
                }
            }
        }
    }
}

}  // namespace laic
