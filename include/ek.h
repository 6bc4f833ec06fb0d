/*
 * ek.h - C ABI of the B200 batch-1 decode megakernel.
 *
 * One call runs one decode step: a single persistent kernel on the caller's
 * stream interprets the per-SM instruction queues built by the Python
 * scheduler. Every buffer is caller-owned device memory passed as a plain
 * pointer. The call is asynchronous, and it allocates nothing once the
 * context's scratch has grown to the model's size (the first call on a
 * context allocates it).
 *
 * Threads: calls on different contexts may come from different host threads
 * at the same time (each call stages its kernel parameters on its own stack;
 * the device-wide set-up is per device and guarded). One context serves one
 * decode step at a time.
 *
 * Errors: a nonzero return is a host-side rejection (bad argument, CUDA launch
 * failure); ek_last_error() describes it. Device-side failures (a cross-SM wait
 * that timed out, a malformed instruction) do not stop the host. The kernel
 * records the first one in the context's status record and drains its queues
 * without further writes. ek_read_status() returns that record.
 */
#ifndef EK_H_
#define EK_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EK_ABI_VERSION 2

/* host return codes */
#define EK_SUCCESS 0
#define EK_E_INVALID 1   /* bad pointer, shape, alignment or size */
#define EK_E_CUDA 2      /* a CUDA runtime call failed */
#define EK_E_UNSUPPORTED 3

/* device status codes (EkStatus.code) */
#define EK_STATUS_OK 0
#define EK_STATUS_TIMEOUT 1         /* a cross-SM counter wait ran out of time */
#define EK_STATUS_BAD_OPCODE 2      /* opcode not defined for this model */
#define EK_STATUS_BAD_INSTRUCTION 3 /* a field of an instruction is out of range */
#define EK_STATUS_RING_TIMEOUT 4    /* internal load ring stalled (engine bug) */
#define EK_STATUS_BAD_COPY 5        /* a weight copy failed its bounds check (engine bug) */

/* cache_flags bits (EkLlamaArgs / EkMixtralArgs) */
#define EK_CACHE_PREFETCH_UPGATE 1   /* L2-prefetch a layer's up/gate rows once the previous layer is done */
#define EK_CACHE_PREFETCH_DOWN 2     /* same for the down-projection rows */
#define EK_CACHE_PREFETCH_BULK 4     /* prefetch with TMA bulk prefetches instead of per-line prefetches */
#define EK_CACHE_PREFETCH_EVICT_LAST 8 /* prefetched lines get evict_last priority */
#define EK_CACHE_WEIGHTS_EVICT_FIRST 16 /* weight loads marked evict_first (read once per step) */
#define EK_CACHE_KV_EVICT_FIRST 32   /* KV-cache loads marked evict_first */

/* EkLlamaArgs.options bits */
/* The last PartialAttention of each KV head to finish merges the head's
 * partials, and the AttentionReduction instructions do nothing. Valid only for
 * schedules whose reductions are terminal over all partials in order (the
 * latency scheduler's); the counters end with the same values. */
#define EK_OPT_FUSE_ATTENTION_REDUCTION 1

typedef struct EkContext EkContext;

/* First device-side failure since the status was last cleared. */
typedef struct EkStatus {
  int32_t code;     /* EK_STATUS_* */
  int32_t sm;       /* queue (thread block) that recorded it */
  int32_t instr;    /* index of the instruction in that queue */
  int32_t opcode;
  int32_t layer;
  int32_t observed; /* counter value last seen (timeouts) */
  int32_t expected; /* counter value waited for (timeouts) / bad word index */
  int32_t detail;   /* timeouts: index of the counter in `barriers` (-1: a tensor-parallel counter
                       in the symmetric buffer); bad instructions: offending word value */
} EkStatus;

/*
 * Arguments of one Llama decode step. The fields are the tensors of
 * `mk_llama(...)`, in the same order (megakernels/demos/latency/mk.py:18-52 and
 * demos/low-latency-llama/llama_1b.cu:23-46 in epic-kernel), plus the model
 * dimensions that the reference compiles into separate binaries.
 * All weights and activations are bf16 unless marked f32.
 */
typedef struct EkLlamaArgs {
  int32_t* barriers;           /* [L, barrier_rows, barrier_cols] int32, zeroed by the caller */
  const int32_t* instructions; /* [num_queues, queue_len, 32] int32 */
  int32_t* timings;            /* [num_queues, queue_len, 128] int32, or NULL */
  const void* qkv_weights;     /* [L, (Hq + 2 Hkv) D, H] */
  const void* attn_ln_weights; /* [L, H] */
  const void* o_weights;       /* [L, H, Hq D] */
  const void* mlp_ln_weights;  /* [L, H] */
  const void* up_weights;      /* [L, I, H] */
  const void* gate_weights;    /* [L, I, H] */
  const void* down_weights;    /* [L, H, I] */
  const void* lm_head_norm_weights; /* [H] */
  const void* lm_head_weights; /* [V, H] */
  void* k_cache;               /* [L, kv_len, Hkv, D] */
  void* v_cache;               /* [L, kv_len, Hkv, D] */
  const float* rope_cos;       /* f32 [rope_rows, D], interleaved pair layout */
  const float* rope_sin;       /* f32 [rope_rows, D] */
  void* hidden_states;         /* [H] */
  void* q_post_rope;           /* [Hq D] */
  void* attn_out;              /* [Hq D] */
  float* attn_lse_intermediates; /* f32 [Hq, max_partials] */
  float* attn_out_intermediates; /* f32 [Hq, max_partials, D] */
  void* silu_out;              /* [I] */
  void* logits;                /* [V] */

  int32_t num_layers, hidden, intermediate, head_dim, num_q_heads, num_kv_heads, vocab;
  int32_t kv_len;        /* cache rows per layer */
  int32_t rope_rows;     /* rows of rope_cos / rope_sin */
  int32_t max_partials;  /* second dim of the attention intermediates */
  int32_t barrier_rows, barrier_cols;
  int32_t num_queues, queue_len;

  int32_t pos_id;
  float attn_scale;
  float rms_norm_eps;
  int32_t skip_attn_reduction;

  int32_t down_reduction_size;  /* columns of W_down per DownProjResidual split (gcd(I, H)) */
  int32_t oproj_reduction_size; /* columns of W_o per O_ProjResidual split (H) */
  int32_t l2_prefetch_stages;   /* >0: stages prefetched into L2 beyond the ring; <0: next instruction's
                                   weights prefetched into L2; 0 = off */
  int32_t record_timings;       /* write timings[q, i, 0..2] when timings != NULL */
  int64_t timeout_ns;           /* bound of every cross-SM wait; <= 0 selects 1 s */
  int32_t cache_flags;          /* EK_CACHE_* bits: L2 eviction hints and MLP-weight L2 prefetch */
  int32_t prefetch_gap_ns;      /* pause of the MLP prefetcher after each 16 KiB it requests (0 = none) */
  int32_t options;              /* EK_OPT_* bits */
  /* Down projections of layers l < deferred_down_layers leave their column-split
   * partial sums for layer l + 1's QKV and O-proj to add into the residual
   * stream (same order and rounding as adding them at once). The instruction
   * stream must then hold layer l + 1's QKV and O-proj instructions; 0 = off. */
  int32_t deferred_down_layers;
  /* Fused token step (all optional, NULL = off). With input_token (int64, one
   * token id) and embed_weights ([vocab, H] bf16), layer 0 reads the token's
   * embedding row instead of hidden_states (which the step then overwrites).
   * With output_token (int64), the index of the largest logit (the first one
   * on ties, as torch.argmax) is written there; lm_head_instructions must then
   * be the number of RMS_LM_Head instructions in the queues. */
  const int64_t* input_token;
  const void* embed_weights;
  int64_t* output_token;
  int32_t lm_head_instructions;
} EkLlamaArgs;

/*
 * Arguments of one Mixtral decode step: the tensors of `mk_mixtral(...)`, in
 * its order (megakernels/mixtral/mk.py:42-96 and the mixtral_globals struct of
 * demos/mixtral/mixtral.cuh:154-203 in epic-kernel), plus model dimensions.
 */
typedef struct EkMixtralArgs {
  int32_t* barriers;           /* [L, barrier_rows, barrier_cols] int32, zeroed by the caller */
  const int32_t* instructions; /* [num_queues, queue_len, 32] int32 */
  int32_t* timings;            /* [num_queues, queue_len, 128] int32, or NULL */
  const void* qkv_weights;     /* [L, (Hq + 2 Hkv) D, H] */
  const void* attn_ln_weights; /* [L, H] */
  const void* o_weights;       /* [L, H, Hq D] */
  const void* expert_gate_weights; /* [L * E, I, H] */
  const void* expert_up_weights;   /* [L * E, I, H] */
  const void* expert_down_weights; /* [L * E, H, I] */
  const void* router_weights;  /* [L * E, H] */
  const void* ffn_ln_weights;  /* [L, H] */
  const void* lm_head_norm_weights; /* [H] */
  const void* lm_head_weights; /* [V, H] */
  void* k_cache;               /* [L, kv_len, Hkv, D] */
  void* v_cache;
  const float* rope_cos;       /* f32 [rope_rows, D] */
  const float* rope_sin;
  void* hidden_states;         /* [H] */
  void* q_post_rope;           /* [Hq D] */
  void* attn_out;              /* [Hq D] */
  float* attn_lse_intermediates; /* f32 [Hq, max_partials] */
  float* attn_out_intermediates; /* f32 [Hq, max_partials, D] */
  void* expert_silu_out;       /* [E, I] */
  void* router_normed_hidden;  /* [H] */
  void* logits;                /* [V], zeroed by the caller (LM-head splits add into it) */
  int32_t* selected_expert_indices; /* int32 [topk] */
  void* selected_expert_scores;     /* bf16 [topk] */
  int32_t* predicted_expert_indices; /* int32 [topk] */

  int32_t num_layers, hidden, intermediate, head_dim, num_q_heads, num_kv_heads, vocab;
  int32_t num_experts, experts_per_token;
  int32_t kv_len, rope_rows, max_partials;
  int32_t barrier_rows, barrier_cols;
  int32_t num_queues, queue_len;

  int32_t pos_id;
  float attn_scale;
  float rms_norm_eps;
  int32_t skip_attn_reduction;

  int32_t l2_prefetch_stages;   /* >0: lookahead L2 prefetch by stages (also speculative expert prefetch);
                                   <0: next instruction's weights; 0 = off */
  int32_t record_timings;
  int64_t timeout_ns;
  int32_t cache_flags;          /* EK_CACHE_* bits (the MLP prefetch bits apply to Llama only) */
  int32_t prefetch_gap_ns;

  /* tensor parallel (after ek_tp_connect): this rank holds num_q_heads /
   * num_kv_heads / intermediate / vocab of its shard; `logits` must be the
   * context's symmetric logits buffer (full vocabulary, vocab * world rows). */
  int32_t tp_lm_instructions;   /* Mixtral_RMS_LM_Head instructions in this rank's queues */
  /* Ring stages (16 KiB) per predicted expert that RmsRouterUpgate's loader
   * prefetches into L2 before the router's choice arrives, once this layer's
   * SpeculativeExpertPredict is done; 0 = off (set it to 0 when the queues hold
   * no SpeculativeExpertPredict). */
  int32_t speculative_prefetch_stages;
} EkMixtralArgs;

/* ABI version compiled into the library (EK_ABI_VERSION). */
int ek_abi_version(void);

/* Message of the last failing host call on this thread ("" if none). */
const char* ek_last_error(void);

/* Create a context on `device` (status record, scratch). One decode step at a
 * time per context. */
int ek_context_create(int device, EkContext** out);
void ek_context_destroy(EkContext* ctx);

/*
 * Llama-3.2 1B / 3B decode step. Replaces the pybind entry points `mk_llama`
 * and `mk_llama_3b` of epic-kernel (demos/low-latency-llama/llama_1b.cu:23-47,
 * llama_3b.cu:26-53; called from megakernels/demos/latency/mk.py:11-52).
 * `stream` is a cudaStream_t (NULL = legacy default stream).
 */
int ek_llama_decode(EkContext* ctx, const EkLlamaArgs* args, void* stream);

/*
 * Llama decode step that allocates nothing, for callers that cannot call
 * cudaMalloc while decoding: runtimes that reserve all device memory up front
 * and hand out only their own pool, or allocators that must not be re-entered
 * from the decode path. This entry point has no counterpart in the reference.
 *
 * The engine's scratch lives in fixed-size device arrays inside this library
 * (about 0.7 MiB per GPU that loads it, kept until process exit): at most
 * 65536 split counters (num_layers * 2 * hidden / 16) and 196608 bf16 partial
 * sums ((hidden / oproj_reduction_size + intermediate / down_reduction_size)
 * * hidden). Larger models are rejected with EK_E_UNSUPPORTED. Runs on the
 * current device; the first call on a device resolves the arrays' addresses,
 * so make it before any stream capture. The arrays are shared by every call on
 * a device: calls that overlap on the GPU race. The status record is cleared
 * at the start of each call; when `status_out` (device memory, may be NULL)
 * is given, the call's EkStatus is copied there on `stream` after the kernel.
 */
int ek_llama_decode_static(const EkLlamaArgs* args, void* stream, EkStatus* status_out);

/*
 * Mixtral-8x7B decode step. Replaces the pybind entry point `mk_mixtral` of
 * epic-kernel (demos/mixtral/mixtral.cu:28-94; called from
 * megakernels/mixtral/mk.py:13-96).
 */
int ek_mixtral_decode(EkContext* ctx, const EkMixtralArgs* args, void* stream);

/*
 * Tensor parallelism for Mixtral (no counterpart in the reference, whose
 * megakernel is single-GPU). Each rank calls ek_tp_setup, which
 * allocates the rank's symmetric buffer (receive slots for the fp32 row
 * partials of O-proj and of the expert down projection, arrival counters, the
 * full-vocabulary logits) and returns its CUDA IPC handle (64 bytes) and the
 * device address of its logits. The handles are exchanged out of band
 * (torch.distributed) and passed, in rank order, to ek_tp_connect. After that,
 * ek_mixtral_decode all-reduces the hidden state inside the kernel: partials
 * are pushed with plain NVLink stores, counters bumped with release.sys
 * atomics, waits are bounded, and every rank sums in rank order, so all ranks
 * hold bit-identical states. A failed launch leaves the counters inconsistent:
 * set up again after one.
 */
int ek_tp_setup(EkContext* ctx, int rank, int world, int num_layers, int hidden, int experts_per_token,
                int full_vocab, void* ipc_handle_out, void** logits_out);
int ek_tp_connect(EkContext* ctx, const void* ipc_handles);

/* Copy the device status record to `out` (synchronises with all work queued
 * on the context's device). With `clear`, reset it to EK_STATUS_OK. */
int ek_read_status(EkContext* ctx, EkStatus* out, int clear);

#ifdef __cplusplus
}
#endif

#endif /* EK_H_ */
