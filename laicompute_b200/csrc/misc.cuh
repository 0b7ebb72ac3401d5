// Small kernels around the decode step: the embedding gather
// (LlamaRuntime::embedding, reference src/inference_v2.cpp:28), position
// bookkeeping, the chained-decode id record and a synthetic KV fill.
#pragma once
#include "common.cuh"
#include "tiles.cuh"
#include "mma_matvec.cuh"  // store_act_record

namespace laic {

struct EmbedParams {
    int type;
    const uint8_t* q;        // token_embd in the fragment-tile layout
    const uint8_t* s;
    int hidden, nb;
    const unsigned* tokens;  // [nseq]
    const int* slots;        // [nseq]
    float* x;                // [nseq][hidden]
    unsigned* counts;        // [max_seqs][vocab] history counts (repeat penalty)
    int vocab;
    // optional: binary16 hi/lo records of x * rec_w for a tile-kernel projection
    uint8_t* rec_out;        // activation records of x * rec_w (rec_off layout)
    const float* rec_w;      // the first rmsnorm weight
    float* ss_out;           // optional: [slices][nseq] sums of x^2 (the next rmsnorm's partials)
    int nseq;
};

// x[s] = row tokens[s] of token_embd; the token joins its slot's history. Grid (nseq,
// slices): CTA (s, y) takes slice y of the row (a multiple of blockDim.x elements) and
// writes its sum of squares to ss_out[y * nseq + s].
__global__ void embed_kernel(const EmbedParams p) {
    __shared__ float red[32];
    const int s = blockIdx.x;
    const int per = ((p.hidden + gridDim.y - 1) / gridDim.y + blockDim.x - 1) / blockDim.x * blockDim.x;
    const int lo = blockIdx.y * per, hi = min(p.hidden, lo + per);
    pdl_wait();
    const unsigned tok = p.tokens[s];
    float ss = 0.f;
    for (int ib = lo; ib < lo + per; ib += blockDim.x) {  // the same trip count in every thread
        const int i = ib + threadIdx.x;
        const bool in = i < hi;
        const float v = in ? tile_value(p.type, p.q, p.s, p.nb, (int)tok, i) : 0.f;
        if (in) p.x[(size_t)s * p.hidden + i] = v;
        if (p.ss_out && in) ss = fmaf(v, v, ss);
        if (p.rec_out && in) store_act_record(p.rec_out, p.nseq, i, s, v * p.rec_w[i]);
    }
    if (p.ss_out) {
        ss = block_sum(ss, red);
        if (threadIdx.x == 0) p.ss_out[(size_t)blockIdx.y * p.nseq + s] = ss;
    }
    if (threadIdx.x == 0 && blockIdx.y == 0)
        atomicAdd(p.counts + (size_t)p.slots[s] * p.vocab + tok, 1u);  // rows may share a slot
    pdl_launch_dependents();
}

// Keeps the stream busy for about `ns` nanoseconds (at most 0.2 s), so that the
// launches queued behind it run back to back instead of waiting on the host.
__global__ void hold_kernel(long long ns) {
    ns = ns < 200000000LL ? ns : 200000000LL;
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    do {
        __nanosleep(1000);
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    } while ((long long)(t - t0) < ns);
}

// Tensor parallel: all-gathered logits [ranks][nseq][vl] -> [nseq][ranks * vl].
__global__ void gather_logits_kernel(const float* g, float* out, int ranks, int nseq, int vl) {
    pdl_wait();
    const long long n = (long long)ranks * nseq * vl;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / vl;
        const int v = (int)(i - t * vl), s = (int)(t % nseq), r = (int)(t / nseq);
        out[((long long)s * ranks + r) * vl + v] = g[i];
    }
}

// End of a prefill step (no sampler): every listed slot moves to the next position.
// Undo a discarded speculative step's bookkeeping: each listed slot's position back to `pos_to`
// and one history count of the token its embedding counted (repeat penalty) taken off.
__global__ void unstep_kernel(const int* slots, const unsigned* toks, const int* pos_to, int* pos, unsigned* counts,
                              int vocab, int nseq) {
    for (int i = threadIdx.x; i < nseq; i += blockDim.x) {
        pos[slots[i]] = pos_to[i];
        atomicSub(counts + (size_t)slots[i] * vocab + toks[i], 1u);
    }
}

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
