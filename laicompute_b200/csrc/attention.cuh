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
#include <cooperative_groups.h>

#include "common.cuh"
#include "mma_matvec.cuh"  // smem_u32, mma16816

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
    int* err;                  // set when a bounded wait runs out (chunked kernel)
    uint8_t* rec_out;          // optional: binary16 hi/lo records of `out` for a tile-kernel projection
    int nseq;                  // sequences of the step (the records' layout)
    const int* npos;           // optional: per query row, its position (batched prefill: causal per row)
    int nbuf;                  // chunk buffers in shared memory (0 or 1: one); a split takes at most
                               // this many chunks when nsplit allows, all fetched before the dependency wait
};

// out[seq][e] = v, plus its activation record when requested.
__device__ __forceinline__ void attn_store(const AttnParams& p, int seq, int e, float v) {
    p.out[(size_t)seq * p.ldo + e] = v;
    if (p.rec_out) store_act_record(p.rec_out, p.nseq, e, seq, v);
}
// attn_store where `live` (every lane of the warp calls it).
__device__ __forceinline__ void attn_emit(const AttnParams& p, int seq, int e, float v, bool live) {
    if (live) attn_store(p, seq, e, v);
}

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
    const int n = (p.npos ? p.npos[seq] : p.pos[slot]) + 1;
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
            attn_store(p, seq, (kvh * G + g) * D + dd, A / L);
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
        attn_store(p, seq, (kvh * G + g) * D + dd, A / L);
    }
    if (threadIdx.x == 0) p.counters[pair] = 0u;
}

// ---------------------------------------------------------------------------
// FP16 KV: tensor-core decode attention over chunks staged in shared memory
// ---------------------------------------------------------------------------
// Grid (nsplit, kv_head, seq). A (sequence, kv head) pair's n = pos + 1
// positions form ceil(n / kAttnChunk) chunks; the first min(nsplit, chunks)
// splits take contiguous runs of them and the rest exit at once, so the work
// follows the live context rather than the capacity.
//
// A chunk's K and V rows (contiguous in the cache) are copied into shared
// memory with 16-byte cp.async, in an XOR-swizzled layout so that ldmatrix
// reads of eight rows hit eight different bank groups. Rows before the newest
// position were written by earlier steps and are fetched before the
// programmatic-dependency wait (overlapping the QKV projection still running);
// the newest row, written by that projection, is fetched after it.
//
// Each warp takes 32 positions of the chunk. The group's G <= 8 query heads
// are the 8 columns of mma.m16n8k16 (fp16 in, fp32 accumulate):
//   scores  S[32 pos][8 heads]  = K q^T   (A = K rows by ldmatrix, B = q)
//   values  O^T[D][8 heads]    += V^T P^T (A = V by ldmatrix.trans, B = p)
// q and p enter as binary16 hi + lo pairs (two products each), which keeps
// them to ~22 significant bits; K and V are the cache's binary16 values.
// Online softmax per head across chunks, then the warps of the CTA and the
// splits are merged with the usual log-sum-exp weights.
constexpr int kAttnChunk = 128;  // positions per chunk: 32 per warp

__host__ __device__ constexpr size_t attn_chunk_smem(int D) { return (size_t)kAttnChunk * D * 2 * 2; }

// element offset of 16-byte column chunk `cc` of row `r` in a swizzled [rows][D] binary16 buffer
template <int D>
__device__ __forceinline__ int attn_swz(int r, int cc) {
    if constexpr (D == 32) return (r * 4 + (cc ^ ((r >> 1) & 3))) * 8;
    else return (r * (D / 8) + (cc ^ (r & 7))) * 8;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// Barrier of the attention warps: the whole CTA of attn_mma_kernel, or the
// four warps of the decode-step kernel that run its attention phase.
__device__ __forceinline__ void attn_group_sync(int id) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kAttnWarps * 32) : "memory");
}

// Largest split count merged inside a thread-block cluster (the portable cluster size).
constexpr int kAttnMaxCluster = 8;

// One split of one (sequence, kv head) pair, run by kAttnWarps warps (tid 0..127)
// on `smem` (attn_chunk_smem(D) bytes per chunk buffer). PDL: fetch older rows
// before the programmatic-dependency wait (standalone kernel); else everything
// after entry. CL: the nsplit CTAs of the pair form one thread-block cluster and
// merge their partials through distributed shared memory (every CTA of the
// cluster reaches both cluster barriers); else the last CTA to finish merges
// them from global scratch (atomic ticket).
template <int D, int GMAX, bool PDL, bool CL = false>
__device__ __forceinline__ void attn_mma_body(const AttnParams& p, int split, int kvh, int seq, uint8_t* smem,
                                              int tid, int bar_id) {
    constexpr int KS = D / 16;  // k-steps of the score product = m-tiles of the value product
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    constexpr int NW = kAttnWarps;
    constexpr int NT = kAttnWarps * 32;
    static_assert(D == 32 || D == 64 || D == 128, "head_dim 32, 64 or 128");
    static_assert(GMAX <= 8, "at most 8 query heads per KV head");
    auto gsync = [&]() { attn_group_sync(bar_id); };
    __half* Ks = reinterpret_cast<__half*>(smem);  // buffer b: K at Ks + b * 2 * chunk * D, then V
    __shared__ __align__(16) __half Ps[NW][2][8][40];  // per warp: p hi/lo [head][position] (rows padded)
    __shared__ float cm[NW][8], cl[NW][8];
    __shared__ int is_last;

    const int lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, c = lane & 3;
    const int G = p.heads / p.kv_heads;

    // positions of this sequence: final for this step before the dependency wait
    const int slot = p.slots[seq];
    const int n = (p.npos ? p.npos[seq] : p.pos[slot]) + 1;
    const int nch = (n + kAttnChunk - 1) / kAttnChunk;
    const int nbuf = max(1, p.nbuf);
    // a context that fits the buffers: one split, no merge; else one chunk per split where
    // nsplit allows (the chunks of a longer split stream through its buffers)
    const int active = nch <= nbuf ? 1 : min(p.nsplit, nch);
    const bool live = split < active;
    if (!live && !CL) {
        if (PDL) pdl_launch_dependents();
        return;
    }
    // (an idle CTA of a cluster has no chunks and an empty partial)
    const int ch0 = live ? split * nch / active : 0, ch1 = live ? (split + 1) * nch / active : 0;
    const __half* kb = reinterpret_cast<const __half*>(p.kc) + (size_t)slot * p.slot_stride + (size_t)kvh * p.cap * D;
    const __half* vb = reinterpret_cast<const __half*>(p.vc) + (size_t)slot * p.slot_stride + (size_t)kvh * p.cap * D;
    // chunk ch lives in buffer (ch - ch0) % nbuf
    auto kbuf = [&](int ch) { return Ks + (size_t)((ch - ch0) % nbuf) * 2 * kAttnChunk * D; };

    // rows [r0, r1) of chunk ch (starting at position c0) into its buffer, all threads
    auto load_rows = [&](int r0, int r1, int ch) {
        __half* kd = kbuf(ch);
        __half* vd = kd + kAttnChunk * D;
        const int c0 = ch * kAttnChunk;
        for (int i = tid; i < (r1 - r0) * CPR; i += NT) {
            const int r = r0 + i / CPR, cc = i % CPR, rl = r - c0;
            cp_async16(kd + attn_swz<D>(rl, cc), kb + (size_t)r * D + cc * 8);
            cp_async16(vd + attn_swz<D>(rl, cc), vb + (size_t)r * D + cc * 8);
        }
        cp_async_commit();
    };
    // value rows past a chunk's end up to the next 32 are read by the last
    // warp's products (with p = 0): make them zeros, not stale bits
    auto zero_tail = [&](int rows, int ch) {
        __half* vd = kbuf(ch) + kAttnChunk * D;
        const int end = min(kAttnChunk, (rows + 31) & ~31);
        for (int i = tid; i < (end - rows) * CPR; i += NT) {
            const int rl = rows + i / CPR, cc = i % CPR;
            *reinterpret_cast<uint4*>(vd + attn_swz<D>(rl, cc)) = make_uint4(0, 0, 0, 0);
        }
    };
    // the first nbuf chunks of this split; PDL: only the rows older than this step's
    for (int ch = ch0; ch < min(ch1, ch0 + nbuf); ++ch) {
        const int c0 = ch * kAttnChunk, c1 = min(n, c0 + kAttnChunk);
        load_rows(c0, PDL ? min(c1, n - 1) : c1, ch);
        zero_tail(c1 - c0, ch);
    }
    if (PDL) {
        pdl_launch_dependents();
        pdl_wait();
        if (ch1 == nch && ch1 - 1 < ch0 + nbuf) load_rows(n - 1, n, ch1 - 1);  // the newest row, after the wait
    }

    // B fragments of the score product: q of head gq (zero past G), scaled by 1/sqrt(d), hi + lo
    uint32_t qh[KS][2], ql[KS][2];
    {
        const float rs = 1.f / p.sqrt_d;
        const float* qg = p.q + (size_t)seq * p.ldq + ((size_t)kvh * G + gq) * D;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int d0 = ks * 16 + 2 * c + 8 * j;
                const float v0 = gq < G ? __ldcg(qg + d0) * rs : 0.f, v1 = gq < G ? __ldcg(qg + d0 + 1) * rs : 0.f;
                const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
                qh[ks][j] = pack_h2(h0, h1);
                ql[ks][j] = pack_h2(__float2half_rn(v0 - __half2float(h0)), __float2half_rn(v1 - __half2float(h1)));
            }
    }

    float m_[2] = {-INFINITY, -INFINITY}, l_[2] = {0.f, 0.f};  // heads 2c, 2c+1
    float o[KS][4];  // O^T: dims (mt*16 + gq, +8) x heads (2c, 2c+1)
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    const int li = lane >> 3, lr = lane & 7;  // ldmatrix: this lane addresses row lr of matrix li

    for (int ch = ch0; ch < ch1; ++ch) {
        const int c0 = ch * kAttnChunk, c1 = min(n, c0 + kAttnChunk);
        const uint32_t ks_a = smem_u32(kbuf(ch)), vs_a = ks_a + kAttnChunk * D * 2;
        cp_async_wait_all();
        gsync();
        const int wp = warp * 32;  // this warp's first row in the chunk
        if (c0 + wp < c1) {
            // ---- scores: two m-tiles of 16 positions
            float s[2][4];
#pragma unroll
            for (int mt2 = 0; mt2 < 2; ++mt2) {
                s[mt2][0] = s[mt2][1] = s[mt2][2] = s[mt2][3] = 0.f;
                const int rr = wp + mt2 * 16 + (li & 1) * 8 + lr;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    uint32_t a[4];
                    ldsm_x4(ks_a + 2 * attn_swz<D>(rr, ks * 2 + (li >> 1)), a);
                    mma16816(s[mt2], a[0], a[1], a[2], a[3], qh[ks][0], qh[ks][1]);
                    mma16816(s[mt2], a[0], a[1], a[2], a[3], ql[ks][0], ql[ks][1]);
                }
            }
            // ---- online softmax per head (this lane: heads 2c and 2c+1)
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int mt2 = 0; mt2 < 2; ++mt2)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int pos = c0 + wp + mt2 * 16 + gq + (e >> 1) * 8;
                    if (pos >= c1) s[mt2][e] = -INFINITY;
                    mx[e & 1] = fmaxf(mx[e & 1], s[mt2][e]);
                }
            float corr[2], sum[2] = {0.f, 0.f};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 4));
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 8));
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 16));
                const float mnew = fmaxf(m_[h], mx[h]);  // finite: the warp has a live position
                corr[h] = expf(m_[h] - mnew);
                m_[h] = mnew;
            }
#pragma unroll
            for (int mt2 = 0; mt2 < 2; ++mt2)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int h = e & 1;
                    const float pv = expf(s[mt2][e] - m_[h]);
                    sum[h] += pv;
                    const int pl = mt2 * 16 + gq + (e >> 1) * 8;
                    const __half hi = __float2half_rn(pv);
                    Ps[warp][0][2 * c + h][pl] = hi;
                    Ps[warp][1][2 * c + h][pl] = __float2half_rn(pv - __half2float(hi));
                }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 4);
                sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 8);
                sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 16);
                l_[h] = l_[h] * corr[h] + sum[h];
            }
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                o[mt][0] *= corr[0]; o[mt][1] *= corr[1];
                o[mt][2] *= corr[0]; o[mt][3] *= corr[1];
            }
            __syncwarp();
            // ---- values: O^T += V^T P^T over two k-steps of 16 positions
#pragma unroll
            for (int kp = 0; kp < 2; ++kp) {
                const uint32_t* ph = reinterpret_cast<const uint32_t*>(&Ps[warp][0][gq][kp * 16 + 2 * c]);
                const uint32_t* pl = reinterpret_cast<const uint32_t*>(&Ps[warp][1][gq][kp * 16 + 2 * c]);
                const uint32_t bh0 = ph[0], bh1 = ph[4], bl0 = pl[0], bl1 = pl[4];  // +4 words = +8 positions
                const int rr = wp + kp * 16 + (li >> 1) * 8 + lr;
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    uint32_t a[4];
                    ldsm_x4_t(vs_a + 2 * attn_swz<D>(rr, mt * 2 + (li & 1)), a);
                    mma16816(o[mt], a[0], a[1], a[2], a[3], bh0, bh1);
                    mma16816(o[mt], a[0], a[1], a[2], a[3], bl0, bl1);
                }
            }
            __syncwarp();
        }
        gsync();  // this chunk's buffer is free
        if (ch + nbuf < ch1) {  // a split longer than its buffers: refill this one
            const int n0 = (ch + nbuf) * kAttnChunk, n1 = min(n, n0 + kAttnChunk);
            load_rows(n0, n1, ch + nbuf);
            zero_tail(n1 - n0, ch + nbuf);
        }
    }

    // ---- merge the warps of this CTA (the chunk buffer holds their accumulators now)
    float* cacc = reinterpret_cast<float*>(smem);  // [NW][8][D]
    if (gq == 0) {
        cm[warp][2 * c] = m_[0]; cm[warp][2 * c + 1] = m_[1];
        cl[warp][2 * c] = l_[0]; cl[warp][2 * c + 1] = l_[1];
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = mt * 16 + gq + (e >> 1) * 8, h = 2 * c + (e & 1);
            cacc[((size_t)warp * 8 + h) * D + d] = o[mt][e];
        }
    gsync();

    const size_t pair = (size_t)seq * p.kv_heads + kvh;
    const int PD = D + 2;
    // per head: the warps' log-sum-exp weights, once
    __shared__ float mw[64][8];  // weights of the warps, then of the splits
    __shared__ float mM[8], mL[8];
    if (tid < G) {
        const int g = tid;
        float M = -INFINITY, L = 0.f;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, cm[w][g]);
        for (int w = 0; w < NW; ++w) {
            const float e = cm[w][g] == -INFINITY ? 0.f : expf(cm[w][g] - M);
            mw[w][g] = e;
            L = fmaf(cl[w][g], e, L);
        }
        mM[g] = M; mL[g] = L;
    }
    gsync();
    __shared__ float cpart[CL ? 8 * D : 1], cpM[8], cpL[8];  // cluster mode: this CTA's partial
    for (int ib = 0; ib < G * D; ib += NT) {  // the same trip count in every thread
        const int i = ib + tid;
        const bool in = i < G * D;
        const int g = in ? i / D : 0, dd = i % D;
        float A = 0.f;
        if (in) {
#pragma unroll
            for (int w = 0; w < NW; ++w) A = fmaf(cacc[((size_t)w * 8 + g) * D + dd], mw[w][g], A);
        }
        if (active == 1) {
            attn_emit(p, seq, kvh * G * D + i, A / mL[g], in && live);
        } else if (!in) {
        } else if (CL) {
            cpart[i] = A;
            if (dd == 0) { cpM[g] = mM[g]; cpL[g] = mL[g]; }
        } else {
            float* dst = p.part + ((pair * p.nsplit + split) * G + g) * PD;
            dst[dd] = A;
            if (dd == 0) { dst[D] = mM[g]; dst[D + 1] = mL[g]; }
        }
    }
    if (active == 1) return;  // the same for every CTA of the pair

    if constexpr (CL) {
        // ---- the splits' partials through distributed shared memory: CTA j of the cluster
        //      is split j; each CTA merges every nsplit-th slice of the elements
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        __shared__ float cw[kAttnMaxCluster][8], cLs[8], rM[kAttnMaxCluster][8], rL[kAttnMaxCluster][8];
        cluster.sync();  // every partial is written
        // every split's (max, sum) per head in one round of remote loads, one thread per pair
        if (tid < active * G) {
            const int j = tid / G, g = tid % G;
            rM[j][g] = *cluster.map_shared_rank(&cpM[g], j);
            rL[j][g] = *cluster.map_shared_rank(&cpL[g], j);
        }
        gsync();
        if (tid < G) {
            const int g = tid;
            float M = -INFINITY, L = 0.f;
            for (int j = 0; j < active; ++j) M = fmaxf(M, rM[j][g]);
            for (int j = 0; j < active; ++j) {
                const float e = rM[j][g] == -INFINITY ? 0.f : expf(rM[j][g] - M);
                cw[j][g] = e;
                L = fmaf(rL[j][g], e, L);
            }
            cLs[g] = L;
        }
        gsync();
        for (int ib = split * NT; ib < G * D; ib += p.nsplit * NT) {
            const int i = ib + tid;
            const bool in = i < G * D;
            const int g = in ? i / D : 0;
            float A = 0.f;
            if (in) {
                float v[kAttnMaxCluster];  // the splits' partials, loaded together, added in split order
#pragma unroll
                for (int j = 0; j < kAttnMaxCluster; ++j) v[j] = j < active ? *cluster.map_shared_rank(&cpart[i], j) : 0.f;
#pragma unroll
                for (int j = 0; j < kAttnMaxCluster; ++j)
                    if (j < active) A = fmaf(v[j], cw[j][g], A);
            }
            attn_emit(p, seq, kvh * G * D + i, A / cLs[g], in);
        }
        cluster.sync();  // no CTA leaves while the others may still read its partial
        return;
    }

    // ---- the last of the active splits merges them (atomic ticket, no spinning)
    __threadfence();
    gsync();
    if (tid == 0) is_last = atomicAdd(p.counters + pair, 1u) == (unsigned)(active - 1);
    gsync();
    if (!is_last) return;
    __threadfence();
    const size_t sstride = (size_t)G * PD;
    const float* base = p.part + pair * p.nsplit * sstride;
    __shared__ float ml[64][8];
    for (int i = tid; i < active * G; i += NT) {  // every split's (max, sum) at once (active <= 64 splits)
        const int j = i / G, g = i % G;
        mw[j][g] = __ldcg(base + j * sstride + g * PD + D);
        ml[j][g] = __ldcg(base + j * sstride + g * PD + D + 1);
    }
    gsync();
    if (tid < G) {  // per head: the splits' weights, in split order
        const int g = tid;
        float M = -INFINITY, L = 0.f;
        for (int j = 0; j < active; ++j) M = fmaxf(M, mw[j][g]);
        for (int j = 0; j < active; ++j) {
            const float e = mw[j][g] == -INFINITY ? 0.f : expf(mw[j][g] - M);
            mw[j][g] = e;
            L = fmaf(ml[j][g], e, L);
        }
        mL[g] = L;
    }
    gsync();
    for (int ib = 0; ib < G * D; ib += NT) {
        const int i = ib + tid;
        const bool in = i < G * D;
        const int g = in ? i / D : 0, dd = i % D;
        const float* src = base + g * PD + dd;
        float A = 0.f;
        int j = 0;
        for (; in && j + 4 <= active; j += 4) {  // four loads in flight, added in split order
            const float v0 = __ldcg(src + j * sstride), v1 = __ldcg(src + (j + 1) * sstride);
            const float v2 = __ldcg(src + (j + 2) * sstride), v3 = __ldcg(src + (j + 3) * sstride);
            A = fmaf(v0, mw[j][g], A);
            A = fmaf(v1, mw[j + 1][g], A);
            A = fmaf(v2, mw[j + 2][g], A);
            A = fmaf(v3, mw[j + 3][g], A);
        }
        for (; in && j < active; ++j) A = fmaf(__ldcg(src + j * sstride), mw[j][g], A);
        attn_emit(p, seq, kvh * G * D + i, A / mL[g], in);
    }
    if (tid == 0) p.counters[pair] = 0u;
}

// CL: launched with a cluster of (nsplit, 1, 1) CTAs, 2 <= nsplit <= kAttnMaxCluster.
template <int D, int GMAX, bool CL>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_mma_kernel(const AttnParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    attn_mma_body<D, GMAX, true, CL>(p, blockIdx.x, blockIdx.y, blockIdx.z, smem, threadIdx.x, 1);
}

}  // namespace laic
