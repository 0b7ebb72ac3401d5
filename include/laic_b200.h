/*
 * laic_b200.h — C ABI of the B200 decode engine for LAICompute's Llama decode loop.
 *
 * The reference has no plugin or FFI layer: its decode path is the C++ class
 * laic::LlamaRuntime (include/laic/inference.hpp:12-34 in the reference), whose
 * private step() (src/inference_v2.cpp:31) and sample() (src/inference_v2.cpp:32)
 * run the per-token forward pass and the token choice on host threads. This
 * header is the device boundary that replaces those two functions: the host
 * surface (include/laic/{gguf,tokenizer,inference}.hpp of this repository)
 * keeps the reference's C++ API and calls these entry points instead of
 * computing on the CPU.
 *
 * Conventions: plain C types, host pointers unless a name says `_dev`, every
 * function returns LAIC_OK (0) or a negative LAIC_E_* code and never throws;
 * laic_last_error() returns the calling thread's last error message.
 */
#ifndef LAIC_B200_H
#define LAIC_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LAIC_API __attribute__((visibility("default")))
#else
#define LAIC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LAIC_OK 0
#define LAIC_E_INVALID (-1)      /* bad argument / shape / state (reference: std::runtime_error) */
#define LAIC_E_CUDA (-2)         /* CUDA runtime or driver failure */
#define LAIC_E_NCCL (-3)         /* collective failure */
#define LAIC_E_CONTEXT (-4)      /* "context length exceeded" (src/inference_v2.cpp:31) */
#define LAIC_E_UNSUPPORTED (-5)  /* type or option this engine does not implement */
#define LAIC_E_MISSING (-6)      /* "missing tensor: ..." (src/gguf.cpp:19) */

/* GGML tensor type codes (reference include/laic/gguf.hpp:9). */
#define LAIC_GGML_F32 0
#define LAIC_GGML_F16 1
#define LAIC_GGML_Q4_0 2
#define LAIC_GGML_Q8_0 8

typedef struct laic_dev laic_dev;
typedef struct laic_tensor laic_tensor;

/* Model architecture: the llama.* GGUF keys LlamaRuntime::load reads
 * (reference src/inference_v2.cpp:27) plus the tokenizer's vocab_size(),
 * which sets the lm_head width (src/inference_v2.cpp:31, end). */
typedef struct laic_dev_desc {
    uint32_t hidden;     /* llama.embedding_length */
    uint32_t layers;     /* llama.block_count */
    uint32_t heads;      /* llama.attention.head_count */
    uint32_t kv_heads;   /* llama.attention.head_count_kv */
    uint32_t ffn;        /* llama.feed_forward_length */
    uint32_t vocab;      /* Gpt2Tokenizer::vocab_size() */
    uint32_t ctx;        /* llama.context_length */
    uint32_t rope_dim;   /* llama.rope.dimension_count */
    float rope_theta;    /* llama.rope.freq_base */
    float rms_eps;       /* llama.attention.layer_norm_rms_epsilon */
} laic_dev_desc;

#define LAIC_FLAG_NO_GRAPH 1u   /* launch kernels one by one instead of replaying a CUDA graph */
#define LAIC_FLAG_NO_PDL 2u     /* no programmatic dependent launch between kernels */
#define LAIC_FLAG_KV_F32 4u     /* FP32 KV cache (the reference's precision) instead of FP16 */
#define LAIC_FLAG_LAYER_LAUNCHES 8u /* one sequence of Q4_0/Q8_0 layers: always launch each projection and
                                      attention separately, never the persistent decode-step kernel */
#define LAIC_FLAG_TRACE 16u     /* the persistent decode-step kernel stamps its phases (laic_dev_step_trace) */
#define LAIC_FLAG_Q4_0_UPSTREAM 128u /* Q4_0 tensors arrive in upstream ggml's nibble order (elements j and
                                        j+16 share byte j); they are reordered to the reference's at upload */
#define LAIC_FLAG_NO_SPECULATION 256u /* laic_dev_step never starts the next step ahead (see laic_dev_step) */
#define LAIC_FLAG_STEP_KERNEL 32u /* one sequence of Q4_0/Q8_0 layers: run each step as the persistent
                                     decode-step kernel where it applies (off by default: per-projection launches
                                     measured faster) */

/* Device-side options (no counterpart in the reference, which is CPU-only). */
typedef struct laic_dev_opts {
    int32_t device;       /* CUDA device ordinal */
    int32_t max_seqs;     /* sequence slots = largest batch of one step */
    int32_t kv_capacity;  /* positions per slot; 0 = ctx */
    int32_t tp_size;      /* tensor-parallel ranks (1 = single GPU) */
    int32_t tp_rank;
    const void* nccl_id;  /* 128-byte ncclUniqueId from laic_nccl_unique_id (tp_size > 1) */
    uint32_t flags;       /* LAIC_FLAG_* */
} laic_dev_opts;

/* GenerationConfig's sampling fields (reference include/laic/inference.hpp:11). */
typedef struct laic_sample_params {
    float temperature;     /* <= 0: greedy argmax (first maximum) */
    uint32_t top_k;        /* 0 = whole vocabulary */
    float top_p;           /* 1 = off */
    float repeat_penalty;  /* 1 = off; applied once per occurrence in the slot's history */
    uint64_t seed;         /* 0 = std::random_device per call, as the reference */
} laic_sample_params;

/* Per-step statistics used by the benchmark's roofline. */
typedef struct laic_dev_stats {
    uint64_t weight_bytes;      /* device bytes of weights read once per full step */
    uint64_t kv_bytes_per_pos;  /* KV bytes written per sequence per step (all layers, K+V) */
    uint32_t launches_per_step; /* kernels in the most recently enqueued full step (chained: incl. the id record) */
    uint32_t launches_per_prefill; /* kernels in the most recently enqueued prefill step */
    uint32_t attn_splits;       /* split-K factor of the last captured step */
    uint32_t tp_size;
} laic_dev_stats;

LAIC_API const char* laic_last_error(void);

/* Engine lifetime. Replaces LlamaRuntime::load's host allocations
 * (src/inference_v2.cpp:27): weights and the KV cache live on the device. */
LAIC_API int laic_dev_create(const laic_dev_desc* desc, const laic_dev_opts* opts, laic_dev** out);
LAIC_API void laic_dev_destroy(laic_dev* dev);

/* Upload one GGUF tensor (name, ggml type, shape ne0-first, raw block bytes as in
 * GgufTensor::data, reference include/laic/gguf.hpp:10). The bytes are copied
 * once; the host buffer is only borrowed for the call. Names follow the
 * reference's lookups: token_embd.weight, output_norm.weight, output.weight,
 * blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,ffn_gate,ffn_up,ffn_down}.weight */
LAIC_API int laic_dev_upload(laic_dev* dev, const char* name, int32_t ggml_type, const uint64_t* shape, int32_t ndim,
                    const void* data, size_t nbytes);

/* One token per listed slot through all layers, without logits or sampling:
 * the prompt loop of generate_ids (src/inference_v2.cpp:34) whose logits are
 * discarded. Advances each slot's position by one. */
LAIC_API int laic_dev_prefill(laic_dev* dev, int32_t nseq, const uint32_t* tokens, const int32_t* slots);

/* The n prompt tokens of one slot in one pass (the KV cache for positions
 * pos..pos+n-1, the slot's position and history advanced): the same effect
 * as n laic_dev_prefill calls, with the projections as dense fp16 tensor-core
 * GEMMs over all n tokens (replaces the per-token prompt loop of
 * LlamaRuntime::generate_ids, reference src/inference_v2.cpp:34). Weights are
 * dequantised to binary16 for it. The FP32-KV parity mode and tensor-parallel
 * engines run the per-token steps instead. */
LAIC_API int laic_dev_prefill_batch(laic_dev* dev, int32_t slot, const uint32_t* tokens, int32_t n);

/* LlamaRuntime::step(token) followed by sample(): one token per listed slot,
 * the full forward pass, then the token choice on the device. `params` holds
 * nparams entries (1 = shared by all sequences, else one per sequence).
 * out_ids[nseq] receives the sampled ids; out_logits (nullable, [nseq][vocab])
 * the raw logits step() would return. Advances each slot's position by one.
 * When a call's tokens are the ids the previous call returned (same slots and
 * sampling parameters), the device starts the following step on those ids
 * before returning; a next call that sends them again only waits for it, any
 * other call (or entry point) first undoes it. Results are the same either way;
 * LAIC_FLAG_NO_SPECULATION turns it off. */
LAIC_API int laic_dev_step(laic_dev* dev, int32_t nseq, const uint32_t* tokens, const int32_t* slots,
                  const laic_sample_params* params, int32_t nparams, uint32_t* out_ids, float* out_logits);

/* Forget a slot's KV cache and token history (generate_ids' cache reset). */
LAIC_API int laic_dev_reset_slot(laic_dev* dev, int32_t slot);
/* Current position (tokens consumed) of a slot. */
LAIC_API int laic_dev_slot_pos(laic_dev* dev, int32_t slot, int64_t* pos);
/* Benchmark helper: fill positions [0, npos) of a slot's KV cache with seeded
 * N(0,1) values and set its position to npos (a long-context cache without
 * running npos prefill steps). */
LAIC_API int laic_dev_fill_kv(laic_dev* dev, int32_t slot, int32_t npos, uint64_t seed);
LAIC_API int laic_dev_sync(laic_dev* dev);
LAIC_API int laic_dev_stats_get(laic_dev* dev, laic_dev_stats* out);
/* The CUDA stream the engine launches on (cudaStream_t as void*). */
LAIC_API void* laic_dev_stream(laic_dev* dev);

/* The reference's decode loop without a host round trip per token: the first
 * token of each listed slot comes from `tokens`, every later step feeds each
 * sequence its own previously sampled id on the device (generate_ids'
 * step(next) -> sample chain, no EOS stop, no callback). Writes
 * out_ids[steps][nseq]; device_ms (nullable) receives the device time of the
 * `steps` step replays measured with CUDA events on the engine stream. */
LAIC_API int laic_dev_decode(laic_dev* dev, int32_t nseq, const uint32_t* tokens, const int32_t* slots,
                             const laic_sample_params* params, int32_t nparams, int32_t steps, uint32_t* out_ids,
                             double* device_ms);

/* Per-kernel-family device time of full steps, for the roofline. */
typedef struct laic_kernel_record {
    char name[16];      /* "embed", "qkv", "attention", "o", "gate_up", "down", "lm_head", "sampler" */
    int32_t launches;   /* launches timed */
    double total_us;    /* summed CUDA-event duration of those launches */
    double bytes;       /* summed algorithmic bytes (weights + activations, or KV read) of those launches */
} laic_kernel_record;

/* Run `steps` full greedy steps of slots 0..nseq-1 (token ids from tokens[steps][nseq])
 * launching kernels one by one with CUDA events around each launch. Each step
 * is queued behind a short stream-holding kernel, so the launches run back to
 * back and the events time the kernels rather than host launch gaps (there is
 * no programmatic overlap between them in this mode). */
LAIC_API int laic_dev_profile(laic_dev* dev, int32_t nseq, const uint32_t* tokens, int32_t steps,
                              laic_kernel_record* out, int32_t max_out, int32_t* n_out);

/* Diagnostics of the persistent one-sequence decode-step kernel (engines created
 * with LAIC_FLAG_TRACE): the globaltimer stamps (ns) of its last launch,
 * out[(cta * phases + phase) * 5 + k] with k = 0 phase start, 1 inputs ready
 * (dependency met, activation records loaded), 2 the CTA's first consumer warp
 * done (attention: before the kv head's ticket), 3 every warp done (attention:
 * after the ticket and any merge of the head), 4 phase done. Phases: 0 the
 * embedding, then per layer QKV, attention, O, gate/up, down, then the lm_head.
 * After those, per CTA and consumer warp 5 counters (ns): waits for a filled
 * ring stage, waits to queue a tile piece, waits for the epilogue warps at
 * the end of a phase, phase waits, and the whole phase loop.
 * No counterpart in the reference. */
LAIC_API int laic_dev_step_trace(laic_dev* dev, uint64_t* out, int64_t max_entries, int64_t* n, int32_t* ctas,
                                 int32_t* phases);

/* Host-only conversion of `n` elements of GGML blocks into the block type the
 * device holds for them (what laic_dev_upload and laic_tensor_create do before
 * the tile repack): Q5_0 becomes Q8_0 with the same scales and int8 values
 * v - 16 (identical values: quant_v2::value, reference src/quant_v2.cpp:12,
 * forms d * (v - 16)); Q4_0 with LAIC_FLAG_Q4_0_UPSTREAM in `flags` is
 * reordered from upstream ggml's nibble order to the reference's
 * (src/quant_v2.cpp:10); F32 / F16 / Q8_0 / Q4_0 are copied. *out_type and
 * *dst_bytes receive the result's type and size; dst == NULL only queries
 * them. Q4_1, Q5_1 and the K-quants are not held on the device
 * (LAIC_E_UNSUPPORTED). No counterpart in the reference. */
LAIC_API int laic_blocks_convert(int32_t ggml_type, const void* src, uint64_t n, uint32_t flags, int32_t* out_type,
                                 void* dst, uint64_t dst_cap, uint64_t* dst_bytes);

/* 128-byte NCCL unique id for laic_dev_opts.nccl_id (rank 0 creates, all ranks share). */
LAIC_API int laic_nccl_unique_id(void* out128);

/* ---- single-tensor entry points (the reference's LlamaRuntime::matvec,
 *      src/inference_v2.cpp:29, and quant_v2::value, src/quant_v2.cpp:8-10) ---- */

/* Upload one [out][in] weight matrix (GGUF shape {in, out}) to `device`. */
LAIC_API int laic_tensor_create(int32_t device, int32_t ggml_type, uint64_t in, uint64_t out, const void* data,
                       size_t nbytes, laic_tensor** t);
LAIC_API void laic_tensor_destroy(laic_tensor* t);
/* y_dev[b][o] = sum_i W[o][i] * x_dev[b][i] for b < batch (FP32 in/out, device pointers). */
LAIC_API int laic_tensor_matvec(laic_tensor* t, const float* x_dev, float* y_dev, int32_t batch, void* stream);
/* out_dev[o*in + i] = decoded W[o][i] (FP32, bit-exact with quant_v2::value). */
LAIC_API int laic_tensor_dequant(laic_tensor* t, float* out_dev, void* stream);
/* Device bytes of the tensor's blocks (the algorithmic bytes of one matvec). */
LAIC_API uint64_t laic_tensor_bytes(laic_tensor* t);

/* Error status of the single-tensor kernels. Their bounded device waits (a
 * bulk copy that never lands, a partial-sum slot never released) do not fault
 * the GPU: they set an error word and the kernel returns, leaving y
 * incomplete. laic_tensor_matvec and laic_tensor_matvec_noalloc return before
 * their kernels run, so they cannot see it; this call synchronises `stream`,
 * reads the word of the tensor's own scratch and of the device's fixed array,
 * clears them and returns LAIC_E_CUDA with the wait's description if either
 * was set (LAIC_OK otherwise). No counterpart in the reference. */
LAIC_API int laic_tensor_check(laic_tensor* t, void* stream);

/* Self-test of the bounded-wait error path on one GPU: runs the tensor-parallel
 * allreduce kernel as rank 0 of two against a peer mailbox that nothing ever
 * writes, with a flag-wait limit of `spin_cycles` SM clocks. The wait runs out,
 * the kernel records its code (4, peer never published) in *code and returns;
 * the call returns LAIC_E_CUDA with that message and the context stays usable.
 * No counterpart in the reference. */
LAIC_API int laic_selftest_peer_timeout(int32_t device, int64_t spin_cycles, int32_t* code);

/* Bytes of the fixed working-memory array behind laic_tensor_matvec_noalloc (per device). */
#define LAIC_FIXED_SCRATCH_BYTES (8u << 20)
/* Same product as laic_tensor_matvec, for hosts that must not allocate device
 * memory once they are serving: the call takes no memory from the CUDA
 * allocator (laic_tensor_matvec grows a per-tensor scratch on demand). Its
 * working memory is one array of LAIC_FIXED_SCRATCH_BYTES compiled into the
 * library; a matrix/batch that needs more returns LAIC_E_INVALID with the size
 * in laic_last_error(). The first call on a device looks up the array's address
 * (setup) and should come before any stream capture; the address is kept for
 * the life of the process, so the library must not be used across a
 * cudaDeviceReset. All calls on a device share the array, which keeps the last
 * call's contents (the split-K tickets, which must start at zero, are cleared
 * on `stream` by every call); calls that overlap in time race on it, so order
 * them on one stream. A device wait that runs out is reported only through
 * laic_tensor_check. No counterpart in the reference, whose matvec runs on the
 * host. */
LAIC_API int laic_tensor_matvec_noalloc(laic_tensor* t, const float* x_dev, float* y_dev, int32_t batch,
                                        void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LAIC_B200_H */
