// Small kernels around the decode step: weight repacking at upload, the
// embedding gather (LlamaRuntime::embedding, reference src/inference_v2.cpp:28),
// position bookkeeping, dequantisation for tests and a synthetic KV fill.
#pragma once
#include "common.cuh"

namespace laic {

// GGUF Q4_0/Q8_0 blocks -> separate planes. Source row r of the chunk goes to
// destination row r * row_mul + row_add (row_mul = 2 interleaves gate/up rows).
// bb = block bytes (18 or 34), qb = quant bytes (16 or 32).
__global__ void repack_blocks_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ qs,
                                     unsigned short* __restrict__ d, long long rows, int nb, int bb, int qb,
                                     int row_mul, long long row_add) {
    const long long total = rows * nb;
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < total;
         b += (long long)gridDim.x * blockDim.x) {
        const long long r = b / nb, c = b % nb;
        const uint8_t* s = src + b * bb;
        const long long dr = r * row_mul + row_add;
        d[dr * nb + c] = (unsigned short)(s[0] | (s[1] << 8));
        uint8_t* q = qs + (dr * nb + c) * qb;
        for (int i = 0; i < qb; i += 2) {
            // two bytes at a time: the source is only 2-byte aligned
            const unsigned short v = (unsigned short)(s[2 + i] | (s[3 + i] << 8));
            *reinterpret_cast<unsigned short*>(q + i) = v;
        }
    }
}

// F16 rows (in halves each): source row r -> destination row r*row_mul + row_add.
__global__ void repack_f16_rows_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long long rows,
                                       int vec_per_row, int row_mul, long long row_add) {
    const long long total = rows * vec_per_row;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / vec_per_row, c = i % vec_per_row;
        dst[(r * row_mul + row_add) * vec_per_row + c] = src[i];
    }
}

// One element of a packed matrix, decoded exactly as quant_v2::value / GgufTensor::value.
__device__ __forceinline__ float packed_value(int type, const void* w, const unsigned short* d, int in, int nb,
                                              long long row, int i) {
    if (type == T_F16) return __half2float(reinterpret_cast<const __half*>(w)[row * in + i]);
    const int c = i >> 5, o = i & 31;
    const float sc = h2f_bits(d[row * nb + c]);
    if (type == T_Q8_0) {
        const int8_t q = reinterpret_cast<const int8_t*>(w)[(row * nb + c) * 32 + o];
        return sc * float(q);
    }
    const uint8_t z = reinterpret_cast<const uint8_t*>(w)[(row * nb + c) * 16 + (o >> 1)];
    return sc * float(((o & 1) ? (z >> 4) : (z & 15)) - 8);
}

__global__ void dequant_kernel(int type, const void* w, const unsigned short* d, int in, int nb, long long rows,
                               float* out) {
    const long long total = rows * in;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x)
        out[e] = packed_value(type, w, d, in, nb, e / in, (int)(e % in));
}

struct EmbedParams {
    int type;
    const void* w;
    const unsigned short* d;
    int hidden, nb;
    const unsigned* tokens;  // [nseq]
    const int* slots;        // [nseq]
    float* x;                // [nseq][hidden]
    unsigned* counts;        // [max_seqs][vocab] history counts (repeat penalty)
    int vocab;
};

// x[s] = row tokens[s] of token_embd; the token joins its slot's history.
__global__ void embed_kernel(const EmbedParams p) {
    const int s = blockIdx.x;
    pdl_wait();
    const unsigned tok = p.tokens[s];
    for (int i = threadIdx.x; i < p.hidden; i += blockDim.x)
        p.x[(size_t)s * p.hidden + i] = packed_value(p.type, p.w, p.d, p.hidden, p.nb, tok, i);
    if (threadIdx.x == 0) p.counts[(size_t)p.slots[s] * p.vocab + tok] += 1u;
    pdl_launch_dependents();
}

// End of a prefill step (no sampler): every listed slot moves to the next position.
__global__ void advance_pos_kernel(const int* slots, int* pos, int nseq) {
    pdl_wait();
    for (int s = threadIdx.x; s < nseq; s += blockDim.x) pos[slots[s]] += 1;
}

// Chained decode: append this step's sampled ids to the history buffer.
__global__ void record_ids_kernel(const unsigned* ids, unsigned* hist, int* counter, int nseq) {
    pdl_wait();
    const int k = *counter;
    for (int s = threadIdx.x; s < nseq; s += blockDim.x) hist[(size_t)k * nseq + s] = ids[s];
    __syncthreads();
    if (threadIdx.x == 0) *counter = k + 1;
}

// Seeded N(0,1) values (Box-Muller on a counter hash) into positions [0, npos)
// of every layer and kv head of one slot, for long-context benchmarks.
__device__ __forceinline__ uint32_t mix32(uint64_t x) {
    x ^= x >> 33; x *= 0xff51afd7ed558ccdULL; x ^= x >> 33; x *= 0xc4ceb9fe1a85ec53ULL; x ^= x >> 33;
    return (uint32_t)x;
}
template <typename KV>
__global__ void fill_kv_kernel(KV* kc, KV* vc, long long layer_stride, long long slot_off, int kv_heads, int cap,
                               int head_dim, int npos, int layers, uint64_t seed) {
    const long long per_layer = (long long)kv_heads * npos * head_dim;
    const long long total = per_layer * layers;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long l = e / per_layer, r = e % per_layer;
        const long long h = r / ((long long)npos * head_dim), t = (r / head_dim) % npos, i = r % head_dim;
        const long long off = l * layer_stride + slot_off + (h * cap + t) * head_dim + i;
        const uint32_t a = mix32(seed * 0x9E3779B97F4A7C15ULL + (uint64_t)e * 2 + 1);
        const uint32_t b = mix32(seed * 0x9E3779B97F4A7C15ULL + (uint64_t)e * 2 + 2);
        const float u1 = (a + 1.f) * 2.3283064e-10f, u2 = b * 2.3283064e-10f;
        const float rad = sqrtf(-2.f * logf(u1));
        float sn, cs;
        sincosf(6.2831853f * u2, &sn, &cs);
        kc[off] = (KV)(rad * cs);
        vc[off] = (KV)(rad * sn);
    }
}

}  // namespace laic
