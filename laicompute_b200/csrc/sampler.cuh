// Token choice on the device: LlamaRuntime::sample (reference src/inference_v2.cpp:32).
//
// One CTA of 1024 threads per sequence, in the reference's order of steps:
//   1. repeat penalty: each occurrence of an id in the slot's history divides a
//      non-negative logit by the penalty, or multiplies a negative one (kept as
//      a per-slot occurrence count, applied count times in sequence);
//   2. temperature <= 0: argmax, first maximum on ties (std::max_element);
//   3. top-k candidates (radix select on order-preserving float keys, ties at
//      the threshold resolved to the lowest ids), sorted by logit descending;
//   4. p = exp((l - max) / T) in float, widened to double, normalised;
//   5. optional top-p over the probability-sorted candidates;
//   6. the inverse-CDF rule of std::discrete_distribution: the first candidate
//      whose cumulative normalised probability is >= u, where u is the draw a
//      freshly seeded mt19937_64 gives (computed on the host per call).
// Steps 4-6 run as the same sequential double recurrences as the reference.
// The only difference from the reference is the candidate ORDER when
// 0 < top_k < vocab and top_p == 1: the reference walks the unspecified order
// std::nth_element leaves; this sampler walks descending-logit order (the
// order the reference itself uses whenever top_p < 1).
// The sampler also advances the slot's position: it is the last kernel of a step.
#pragma once
#include "common.cuh"

namespace laic {

struct SampleDev {
    float temperature;
    unsigned top_k;
    float top_p;
    float repeat_penalty;
    double u;  // uniform draw of std::discrete_distribution, in [0, 1)
};

struct SamplerParams {
    const float* logits;   // [nseq][ldl]
    int ldl, vocab;
    const int* slots;      // [nseq]
    const unsigned* counts;  // [max_seqs][vocab] occurrences in each slot's history
    const SampleDev* sp;   // [nparams]
    int nparams;
    unsigned* out_ids;     // [nseq]
    unsigned* next_tokens; // [nseq] the sampled id is also the next step's input token
    int* pos;              // [max_seqs]
    int* err;              // set to 1 when a request exceeds the sampler's candidate limit
    // grid.y > 1 (few sequences): each CTA takes a slice of the vocabulary for the argmax, the
    // last to finish (atomic ticket) combines the slices and runs the rest for the sequence
    float* part_v;         // [nseq][grid.y] slice maxima (scratch)
    int* part_i;           // [nseq][grid.y] their ids
    unsigned* part_cnt;    // [nseq] tickets, zero between launches
};

constexpr int kSampleThreads = 1024;
constexpr int kSampleSlices = 16;  // CTAs per sequence for the argmax when a step has few sequences
constexpr int kMaxCand = 1024;

__device__ __forceinline__ float penalized(float l, unsigned c, float rp) {
    for (unsigned i = 0; i < c; ++i) l = l >= 0.f ? l / rp : l * rp;
    return l;
}
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive block scan of one int per thread (1024 threads); returns the total.
__device__ __forceinline__ int block_excl_scan(int v, int* buf, int& excl) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) buf[w] = x;
    __syncthreads();
    if (w == 0) {
        int t = buf[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        buf[lane] = t;
    }
    __syncthreads();
    excl = x - v + (w > 0 ? buf[w - 1] : 0);
    const int total = buf[31];
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SamplerParams p) {
    __shared__ float cv[kMaxCand];
    __shared__ int ci[kMaxCand];
    __shared__ double cp[kMaxCand];
    __shared__ int hist[256];
    __shared__ int scan_buf[32];
    __shared__ float redv[32];
    __shared__ int redi[32];
    __shared__ uint32_t sh_prefix;
    __shared__ int sh_krem;
    __shared__ int sh_err;

    const int seq = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int V = p.vocab;

    pdl_wait();
    const SampleDev sp = p.sp[p.nparams == 1 ? 0 : seq];
    const int slot = p.slots[seq];
    const float* lg = p.logits + (size_t)seq * p.ldl;
    const unsigned* cnt = p.counts + (size_t)slot * V;
    const bool pen = sp.repeat_penalty != 1.f;
    auto L = [&](int i) { return pen ? penalized(lg[i], cnt[i], sp.repeat_penalty) : lg[i]; };

    // block argmax with lowest index on ties; also the maximum for the softmax.
    // Each thread walks its indices in increasing order (four per float4, several
    // float4 loads in flight), so a strict > keeps its first maximum.
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    auto consider = [&](float v, int i) {
        if (v > bv || bi == 0x7fffffff) { bv = v; bi = i; }
    };
    const bool vec = (V % 4 == 0) && (p.ldl % 4 == 0);
    const int P = gridDim.y;
    if (vec) {
        const float4* lg4 = reinterpret_cast<const float4*>(lg);
        const uint4* cn4 = reinterpret_cast<const uint4*>(cnt);
        const int V4 = V / 4;
        const int per = (V4 + P - 1) / P, f_lo = blockIdx.y * per, f_hi = min(V4, f_lo + per);
#pragma unroll 8
        for (int i4 = f_lo + tid; i4 < f_hi; i4 += kSampleThreads) {
            float4 v = lg4[i4];
            if (pen) {
                const uint4 c = cn4[i4];
                v.x = penalized(v.x, c.x, sp.repeat_penalty); v.y = penalized(v.y, c.y, sp.repeat_penalty);
                v.z = penalized(v.z, c.z, sp.repeat_penalty); v.w = penalized(v.w, c.w, sp.repeat_penalty);
            }
            consider(v.x, 4 * i4); consider(v.y, 4 * i4 + 1); consider(v.z, 4 * i4 + 2); consider(v.w, 4 * i4 + 3);
        }
    } else {
        const int per = (V + P - 1) / P, e_lo = blockIdx.y * per, e_hi = min(V, e_lo + per);
        for (int i = e_lo + tid; i < e_hi; i += kSampleThreads) consider(L(i), i);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { redv[w] = bv; redi[w] = bi; }
    if (tid == 0) sh_err = 0;
    __syncthreads();
    if (w == 0) {
        bv = redv[lane]; bi = redi[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { redv[0] = bv; redi[0] = bi; }
    }
    __syncthreads();
    if (P > 1) {  // this slice's maximum; the last CTA of the sequence goes on with all of them
        __shared__ int sh_last;
        if (tid == 0) {
            p.part_v[(size_t)seq * P + blockIdx.y] = redv[0];
            p.part_i[(size_t)seq * P + blockIdx.y] = redi[0];
            __threadfence();
            sh_last = atomicAdd(p.part_cnt + seq, 1u) == (unsigned)(P - 1);
        }
        __syncthreads();
        if (!sh_last) return;
        if (tid == 0) {
            __threadfence();
            float v = -INFINITY;
            int id = 0x7fffffff;
            for (int y = 0; y < P; ++y) {  // slices in id order: a strict > keeps the first maximum
                const float vy = __ldcg(p.part_v + (size_t)seq * P + y);
                const int iy = __ldcg(p.part_i + (size_t)seq * P + y);
                if (iy != 0x7fffffff && (vy > v || id == 0x7fffffff)) { v = vy; id = iy; }
            }
            redv[0] = v;
            redi[0] = id;
            p.part_cnt[seq] = 0u;
        }
        __syncthreads();
    }
    const float vmax = redv[0];
    const int imax = redi[0];

    if (sp.temperature <= 0.f) {
        if (tid == 0) { p.out_ids[seq] = p.next_tokens[seq] = (unsigned)imax; p.pos[slot] += 1; }
        return;
    }

    // ---- candidate set
    int k = (sp.top_k == 0 || (int)sp.top_k >= V) ? V : (int)sp.top_k;
    const bool full = k == V;
    const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
    const int lo = min(V, tid * chunk), hi = min(V, lo + chunk);

    __shared__ double dsum[kSampleThreads];
    double full_total = 0.0;
    if (full) {
        // whole-vocabulary mass: per-thread contiguous chunks, then an inclusive scan
        double s = 0.0;
        for (int i = lo; i < hi; ++i) s += (double)expf((L(i) - vmax) / sp.temperature);
        dsum[tid] = s;
        __syncthreads();
        for (int o = 1; o < kSampleThreads; o <<= 1) {
            const double y = tid >= o ? dsum[tid - o] : 0.0;
            __syncthreads();
            dsum[tid] += y;
            __syncthreads();
        }
        full_total = dsum[kSampleThreads - 1];
    }
    if (full && sp.top_p >= 1.f) {
        // whole vocabulary in index order: the first id whose cumulative mass reaches
        // u * total (the reference's two double normalisations fold into u)
        const double target = sp.u * full_total;
        const double before = tid > 0 ? dsum[tid - 1] : 0.0, after = dsum[tid];
        if (before < target && target <= after) {
            double acc = before;
            int pick = hi - 1;
            for (int i = lo; i < hi; ++i) {
                acc += (double)expf((L(i) - vmax) / sp.temperature);
                if (acc >= target) { pick = i; break; }
            }
            p.out_ids[seq] = (unsigned)pick;
        }
        __syncthreads();
        if (tid == 0) {
            if (target <= 0.0) p.out_ids[seq] = 0u;
            p.next_tokens[seq] = p.out_ids[seq];
            p.pos[slot] += 1;
        }
        return;
    }
    if (full) k = kMaxCand <= V ? kMaxCand : V;  // top-p over the whole vocabulary: widest candidate set
    if (k > kMaxCand) {
        if (tid == 0) { *p.err = 1; p.out_ids[seq] = p.next_tokens[seq] = (unsigned)imax; p.pos[slot] += 1; }
        return;
    }

    // radix select of the k-th largest key (4 passes of 8 bits)
    if (tid == 0) { sh_prefix = 0u; sh_krem = k; }
    __syncthreads();
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        const uint32_t prefix = sh_prefix;
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = order_key(L(i));
            if (pass == 0 || (key >> (shift + 8)) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
        }
        __syncthreads();
        if (tid == 0) {
            int krem = sh_krem, above = 0, b = 255;
            for (; b > 0; --b) {
                if (above + hist[b] >= krem) break;
                above += hist[b];
            }
            sh_prefix = (prefix << 8) | (uint32_t)b;
            sh_krem = krem - above;
        }
        __syncthreads();
    }
    const uint32_t thr = sh_prefix;
    const int need_ties = sh_krem;  // ties at thr to take (lowest ids first)

    // ordered compaction: ids with key > thr, then the first need_ties ids with key == thr
    int ngt = 0, neq = 0;
    for (int i = lo; i < hi; ++i) {
        const uint32_t key = order_key(L(i));
        ngt += key > thr;
        neq += key == thr;
    }
    int ogt, oeq;
    const int tot_gt = block_excl_scan(ngt, scan_buf, ogt);
    block_excl_scan(neq, scan_buf, oeq);
    for (int i = lo; i < hi; ++i) {
        const float v = L(i);
        const uint32_t key = order_key(v);
        if (key > thr) { cv[ogt] = v; ci[ogt] = i; ++ogt; }
        else if (key == thr) {
            if (oeq < need_ties) { cv[tot_gt + oeq] = v; ci[tot_gt + oeq] = i; }
            ++oeq;
        }
    }
    // pad to a power of two and bitonic-sort by (logit desc, id asc)
    int np2 = 1;
    while (np2 < k) np2 <<= 1;
    for (int i = k + tid; i < np2; i += kSampleThreads) { cv[i] = -INFINITY; ci[i] = 0x7fffffff; }
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < np2; i += kSampleThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc_blk = (i & size) == 0;
                    const float a = cv[i], b = cv[j];
                    const int ia = ci[i], ib = ci[j];
                    const bool a_first = a > b || (a == b && ia < ib);
                    if (desc_blk ? !a_first : a_first) { cv[i] = b; cv[j] = a; ci[i] = ib; ci[j] = ia; }
                }
            }
            __syncthreads();
        }
    }
    // probabilities (parallel), then the reference's sequential double recurrences
    const float mx = cv[0];
    for (int j = tid; j < k; j += kSampleThreads) cp[j] = (double)expf((cv[j] - mx) / sp.temperature);
    __syncthreads();
    if (tid == 0) {
        double sum = 0.0;
        if (full) sum = full_total;  // candidates are the head of the whole vocabulary
        else for (int j = 0; j < k; ++j) sum += cp[j];
        for (int j = 0; j < k; ++j) cp[j] /= sum;
        int kk = k;
        if (sp.top_p < 1.f) {
            double acc = 0.0;
            int keep = 0;
            for (int j = 0; j < k; ++j) { acc += cp[j]; keep++; if (acc >= (double)sp.top_p) break; }
            if (full && acc < (double)sp.top_p && k < V) sh_err = 1;  // mass beyond the candidate limit
            double ns = 0.0;
            for (int j = 0; j < keep; ++j) ns += cp[j];
            for (int j = 0; j < keep; ++j) cp[j] /= ns;
            kk = keep;
        }
        int pick = 0;
        if (kk >= 2) {
            double s2 = 0.0;
            for (int j = 0; j < kk; ++j) s2 += cp[j];
            double c = 0.0;
            pick = kk - 1;
            for (int j = 0; j < kk; ++j) {
                c += cp[j] / s2;
                const double cj = j == kk - 1 ? 1.0 : c;
                if (cj >= sp.u) { pick = j; break; }
            }
        }
        p.out_ids[seq] = p.next_tokens[seq] = (unsigned)ci[pick];
        if (sh_err) *p.err = 1;
        p.pos[slot] += 1;
    }
}

}  // namespace laic
