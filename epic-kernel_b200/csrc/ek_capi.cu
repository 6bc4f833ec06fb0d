// C ABI of the decode engine (include/ek.h): contexts, argument validation,
// TMA tensor-map encoding and the device status record.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ek.h"
#include "ek_launch.h"

using ek::KParams;

struct EkContext {
  int device = 0;
  ek::DevStatus* status = nullptr;
  unsigned* counters = nullptr;
  size_t counters_cap = 0;  // elements
  __nv_bfloat16* partials = nullptr;
  size_t partials_cap = 0;  // elements
  unsigned epoch = 0;
  // Mixtral tensor parallelism
  int tp_world = 1, tp_rank = 0;
  int tp_layers = 0, tp_hidden = 0, tp_topk = 0, tp_vocab = 0;
  char* tp_buf = nullptr;
  size_t tp_bytes = 0;
  char* tp_peer[ek::MAX_TP] = {};
  bool tp_connected = false;
  unsigned tp_step = 0;
  long long off_recv_o = 0, off_recv_d = 0, off_cnt_o = 0, off_cnt_d = 0, off_cnt_lm = 0, off_logits = 0;
};

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(EK_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 tensor map of a KV cache [L*T, Hkv, D], box D x 1 head x tk tokens.
int encode_kv(CUtensorMap* m, const void* base, long long rows, int hkv, int d, int tk,
              const char* name) {
  EncodeTiledFn enc = get_encoder();
  if (!enc) return fail(EK_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)hkv, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)hkv * d * 2};
  cuuint32_t box[3] = {(cuuint32_t)d, 1, (cuuint32_t)tk};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EK_E_INVALID, "tensor map for %s failed (CUresult %d)", name, (int)r);
  return EK_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int grow(EkContext* ctx, size_t counters, size_t partials) {
  cudaError_t e;
  if (counters > ctx->counters_cap) {
    if (ctx->counters) cudaFree(ctx->counters);
    ctx->counters = nullptr;
    ctx->counters_cap = 0;
    if ((e = cudaMalloc(&ctx->counters, counters * sizeof(unsigned))) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(split counters)");
    if ((e = cudaMemset(ctx->counters, 0, counters * sizeof(unsigned))) != cudaSuccess)
      return cuda_fail(e, "cudaMemset(split counters)");
    ctx->counters_cap = counters;
  }
  if (partials > ctx->partials_cap) {
    if (ctx->partials) cudaFree(ctx->partials);
    ctx->partials = nullptr;
    ctx->partials_cap = 0;
    if ((e = cudaMalloc(&ctx->partials, partials * 2)) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(split partials)");
    ctx->partials_cap = partials;
  }
  return EK_SUCCESS;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" {

int ek_abi_version(void) { return EK_ABI_VERSION; }

const char* ek_last_error(void) { return g_err.c_str(); }

int ek_context_create(int device, EkContext** out) {
  if (!out) return fail(EK_E_INVALID, "out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(EK_E_INVALID, "device %d out of range (%d devices)", device, n);
  DeviceGuard g(device);
  EkContext* ctx = new EkContext();
  ctx->device = device;
  if ((e = cudaMalloc(&ctx->status, sizeof(ek::DevStatus))) != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "cudaMalloc(status)");
  }
  if ((e = cudaMemset(ctx->status, 0, sizeof(ek::DevStatus))) != cudaSuccess) {
    cudaFree(ctx->status);
    delete ctx;
    return cuda_fail(e, "cudaMemset(status)");
  }
  *out = ctx;
  return EK_SUCCESS;
}

void ek_context_destroy(EkContext* ctx) {
  if (!ctx) return;
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  if (ctx->status) cudaFree(ctx->status);
  if (ctx->counters) cudaFree(ctx->counters);
  if (ctx->partials) cudaFree(ctx->partials);
  for (int r = 0; r < ctx->tp_world; ++r)
    if (ctx->tp_peer[r] && r != ctx->tp_rank) cudaIpcCloseMemHandle(ctx->tp_peer[r]);
  if (ctx->tp_buf) cudaFree(ctx->tp_buf);
  delete ctx;
}

static long long align256(long long x) { return (x + 255) & ~255ll; }

int ek_tp_setup(EkContext* ctx, int rank, int world, int num_layers, int hidden, int experts_per_token,
                int full_vocab, void* ipc_handle_out, void** logits_out) {
  if (!ctx || !ipc_handle_out || !logits_out) return fail(EK_E_INVALID, "NULL argument");
  if (world < 2 || world > ek::MAX_TP || rank < 0 || rank >= world)
    return fail(EK_E_INVALID, "rank %d / world %d (2..%d ranks)", rank, world, ek::MAX_TP);
  if (num_layers < 1 || hidden < 16 || hidden % 16 || experts_per_token < 1 || full_vocab < 16)
    return fail(EK_E_INVALID, "bad dims");
  DeviceGuard g(ctx->device);
  if (ctx->tp_buf) {
    for (int r = 0; r < ctx->tp_world; ++r)
      if (ctx->tp_peer[r] && r != ctx->tp_rank) cudaIpcCloseMemHandle(ctx->tp_peer[r]);
    cudaFree(ctx->tp_buf);
    ctx->tp_buf = nullptr;
  }
  long long off = 0;
  ctx->off_recv_o = off; off = align256(off + (long long)world * hidden * 4);
  ctx->off_recv_d = off; off = align256(off + (long long)world * experts_per_token * hidden * 4);
  ctx->off_cnt_o = off; off = align256(off + (long long)num_layers * (hidden / 16) * 4);
  ctx->off_cnt_d = off; off = align256(off + (long long)num_layers * (hidden / 16) * 4);
  ctx->off_cnt_lm = off; off = align256(off + 16);
  ctx->off_logits = off; off = align256(off + (long long)full_vocab * 2);
  cudaError_t e;
  if ((e = cudaMalloc(&ctx->tp_buf, off)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(tp buffer)");
  if ((e = cudaMemset(ctx->tp_buf, 0, off)) != cudaSuccess) return cuda_fail(e, "cudaMemset(tp buffer)");
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, ctx->tp_buf)) != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  std::memcpy(ipc_handle_out, &h, 64);
  *logits_out = ctx->tp_buf + ctx->off_logits;
  ctx->tp_bytes = off;
  ctx->tp_world = world;
  ctx->tp_rank = rank;
  ctx->tp_layers = num_layers;
  ctx->tp_hidden = hidden;
  ctx->tp_topk = experts_per_token;
  ctx->tp_vocab = full_vocab;
  ctx->tp_connected = false;
  ctx->tp_step = 0;
  for (int r = 0; r < ek::MAX_TP; ++r) ctx->tp_peer[r] = nullptr;
  return EK_SUCCESS;
}

int ek_tp_connect(EkContext* ctx, const void* ipc_handles) {
  if (!ctx || !ipc_handles) return fail(EK_E_INVALID, "NULL argument");
  if (!ctx->tp_buf) return fail(EK_E_INVALID, "ek_tp_setup first");
  DeviceGuard g(ctx->device);
  const char* hs = static_cast<const char*>(ipc_handles);
  for (int r = 0; r < ctx->tp_world; ++r) {
    if (r == ctx->tp_rank) {
      ctx->tp_peer[r] = ctx->tp_buf;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + 64 * r, 64);
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    ctx->tp_peer[r] = static_cast<char*>(ptr);
  }
  ctx->tp_connected = true;
  ctx->tp_step = 0;
  return EK_SUCCESS;
}

int ek_read_status(EkContext* ctx, EkStatus* out, int clear) {
  if (!ctx || !out) return fail(EK_E_INVALID, "NULL argument");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  ek::DevStatus s;
  if ((e = cudaMemcpy(&s, ctx->status, sizeof(s), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpy(status)");
  static_assert(sizeof(EkStatus) == 8 * sizeof(int32_t), "EkStatus layout");
  std::memcpy(out, &s, sizeof(EkStatus));
  if (clear && (e = cudaMemset(ctx->status, 0, sizeof(ek::DevStatus))) != cudaSuccess)
    return cuda_fail(e, "cudaMemset(status)");
  return EK_SUCCESS;
}

int ek_llama_decode(EkContext* ctx, const EkLlamaArgs* a, void* stream) {
  if (!ctx || !a) return fail(EK_E_INVALID, "NULL context or arguments");
  const void* required[] = {a->barriers, a->instructions, a->qkv_weights, a->attn_ln_weights,
                            a->o_weights, a->mlp_ln_weights, a->up_weights, a->gate_weights,
                            a->down_weights, a->lm_head_norm_weights, a->lm_head_weights,
                            a->k_cache, a->v_cache, a->rope_cos, a->rope_sin, a->hidden_states,
                            a->q_post_rope, a->attn_out, a->attn_lse_intermediates,
                            a->attn_out_intermediates, a->silu_out, a->logits};
  for (size_t i = 0; i < sizeof(required) / sizeof(required[0]); ++i) {
    if (!required[i]) return fail(EK_E_INVALID, "pointer argument %zu is NULL", i);
    if (!aligned16(required[i])) return fail(EK_E_INVALID, "pointer argument %zu is not 16-byte aligned", i);
  }
  if (a->timings && !aligned16(a->timings)) return fail(EK_E_INVALID, "timings is not 16-byte aligned");

  const int L = a->num_layers, H = a->hidden, I = a->intermediate, D = a->head_dim;
  const int Hq = a->num_q_heads, Hkv = a->num_kv_heads, V = a->vocab;
  if (L < 1 || H < 256 || I < 256 || V < 16 || Hq < 1 || Hkv < 1)
    return fail(EK_E_INVALID, "bad model dims L=%d H=%d I=%d V=%d Hq=%d Hkv=%d", L, H, I, V, Hq, Hkv);
  if (D != 64 && D != 128) return fail(EK_E_UNSUPPORTED, "head_dim %d (supported: 64, 128)", D);
  if (H % 256 || I % 256) return fail(EK_E_INVALID, "hidden and intermediate must be multiples of 256");
  if (V % 16) return fail(EK_E_INVALID, "vocab %d not a multiple of 16", V);
  if (Hq % Hkv) return fail(EK_E_INVALID, "num_q_heads %% num_kv_heads != 0");
  if (Hq * D != H) return fail(EK_E_INVALID, "num_q_heads * head_dim (%d) != hidden (%d)", Hq * D, H);
  const int gqa = Hq / Hkv;
  if (gqa > ek::MAX_GQA || ek::CW * gqa * (D + 2) * 4 > ek::ACT_BYTES)
    return fail(EK_E_UNSUPPORTED, "GQA ratio %d too large for head_dim %d", gqa, D);
  const int dR = a->down_reduction_size > 0 ? a->down_reduction_size : I;
  const int oR = a->oproj_reduction_size > 0 ? a->oproj_reduction_size : H;
  if (dR % 256 || I % dR || I / dR > 255)
    return fail(EK_E_INVALID, "down_reduction_size %d must be a multiple of 256 dividing %d", dR, I);
  if (oR % 256 || H % oR || H / oR > 255)
    return fail(EK_E_INVALID, "oproj_reduction_size %d must be a multiple of 256 dividing %d", oR, H);
  if (H * 2 > ek::ACT_BYTES || dR * 2 > ek::ACT_BYTES)
    return fail(EK_E_UNSUPPORTED, "activation vector does not fit in shared memory");
  if (a->kv_len < 1 || a->rope_rows < 1 || a->max_partials < 1)
    return fail(EK_E_INVALID, "kv_len, rope_rows and max_partials must be positive");
  if (a->pos_id < 0 || a->pos_id >= a->kv_len || a->pos_id >= a->rope_rows)
    return fail(EK_E_INVALID, "pos_id %d outside the KV cache (%d) or rope table (%d)", a->pos_id,
                a->kv_len, a->rope_rows);
  if (a->barrier_rows < 6 || a->barrier_cols < Hq + 2 * Hkv)
    return fail(EK_E_INVALID, "barriers must be at least [L, 6, Hq + 2 Hkv]");
  if (a->queue_len < 1 || a->num_queues < 1) return fail(EK_E_INVALID, "empty instruction tensor");

  DeviceGuard g(ctx->device);
  int nsm = 0;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, ctx->device);
  if (a->num_queues > nsm)
    return fail(EK_E_INVALID, "%d instruction queues but only %d SMs", a->num_queues, nsm);

  const size_t nctr = (size_t)L * 2 * (H / 16);
  const size_t npart = (size_t)(H / oR + I / dR) * H;
  int rc = grow(ctx, nctr, npart);
  if (rc) return rc;

  KParams p;  // per call (thread-safe); the launch copies it into the kernel parameters
  std::memset(&p, 0, sizeof(p));
  const int qkv_rows = (Hq + 2 * Hkv) * D;
  const int tk = ek::HALF_STAGE / (D * 2);
  if ((rc = encode_kv(&p.tm_k, a->k_cache, (long long)L * a->kv_len, Hkv, D, tk, "k_cache"))) return rc;
  if ((rc = encode_kv(&p.tm_v, a->v_cache, (long long)L * a->kv_len, Hkv, D, tk, "v_cache"))) return rc;

  p.w_qkv = static_cast<const __nv_bfloat16*>(a->qkv_weights);
  p.w_o = static_cast<const __nv_bfloat16*>(a->o_weights);
  p.w_up = static_cast<const __nv_bfloat16*>(a->up_weights);
  p.w_gate = static_cast<const __nv_bfloat16*>(a->gate_weights);
  p.w_down = static_cast<const __nv_bfloat16*>(a->down_weights);
  p.w_lm = static_cast<const __nv_bfloat16*>(a->lm_head_weights);
  p.rows_qkv = (long long)L * qkv_rows;
  p.rows_o = (long long)L * H;
  p.rows_up = (long long)L * I;
  p.rows_down = (long long)L * H;
  p.rows_lm = V;
  p.barriers = a->barriers;
  p.instructions = a->instructions;
  p.timings = a->timings;
  p.attn_ln = static_cast<const __nv_bfloat16*>(a->attn_ln_weights);
  p.mlp_ln = static_cast<const __nv_bfloat16*>(a->mlp_ln_weights);
  p.lm_norm = static_cast<const __nv_bfloat16*>(a->lm_head_norm_weights);
  p.k_cache = static_cast<__nv_bfloat16*>(a->k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(a->v_cache);
  p.rope_cos = a->rope_cos;
  p.rope_sin = a->rope_sin;
  p.hidden = static_cast<__nv_bfloat16*>(a->hidden_states);
  p.q = static_cast<__nv_bfloat16*>(a->q_post_rope);
  p.attn_out = static_cast<__nv_bfloat16*>(a->attn_out);
  p.lse = a->attn_lse_intermediates;
  p.attn_o = a->attn_out_intermediates;
  p.silu = static_cast<__nv_bfloat16*>(a->silu_out);
  p.logits = static_cast<__nv_bfloat16*>(a->logits);
  p.status = ctx->status;
  p.split_counters = ctx->counters;
  p.split_partials = ctx->partials;
  p.L = L; p.H = H; p.I = I; p.D = D; p.Hq = Hq; p.Hkv = Hkv; p.V = V;
  p.T = a->kv_len; p.rope_rows = a->rope_rows; p.maxP = a->max_partials;
  p.brow = a->barrier_rows; p.bcol = a->barrier_cols;
  p.nq = a->num_queues; p.Q = a->queue_len;
  p.qkv_rows = qkv_rows; p.gqa = gqa; p.tk = tk;
  p.pos = a->pos_id; p.skip_red = a->skip_attn_reduction ? 1 : 0;
  p.scale = a->attn_scale; p.eps = a->rms_norm_eps;
  p.down_R = dR; p.o_R = oR; p.down_splits = I / dR; p.o_splits = H / oR;
  p.model = ek::MODEL_LLAMA;
  p.down_done_target = (I / dR) * (H / 16);
  p.defer_down = (I / dR > 1 && H / oR == 1) ? min(max(a->deferred_down_layers, 0), L - 1) : 0;
  p.fuse_red = (a->options & EK_OPT_FUSE_ATTENTION_REDUCTION) ? 1 : 0;
  if (p.fuse_red && p.gqa * a->max_partials > ek::MAX_GQA * 160)
    return fail(EK_E_UNSUPPORTED, "fused attention reduction: %d heads x %d partials", p.gqa, a->max_partials);
  p.pf_stages = a->l2_prefetch_stages > 0 ? a->l2_prefetch_stages : 0;
  p.pf_next = a->l2_prefetch_stages < 0 ? min(-a->l2_prefetch_stages, 2) : 0;
  p.pf_mlp = a->cache_flags;
  p.pf_gap_ns = a->prefetch_gap_ns > 0 ? (unsigned)a->prefetch_gap_ns : 0u;
  p.record = a->record_timings && a->timings ? 1 : 0;
  p.timeout_ns = a->timeout_ns > 0 ? a->timeout_ns : 1000000000ll;
  if (a->output_token && a->lm_head_instructions < 1)
    return fail(EK_E_INVALID, "output_token needs lm_head_instructions >= 1");
  if ((a->input_token == nullptr) != (a->embed_weights == nullptr))
    return fail(EK_E_INVALID, "input_token and embed_weights go together");
  if (a->embed_weights && !aligned16(a->embed_weights)) return fail(EK_E_INVALID, "embed_weights not 16-byte aligned");
  p.in_token = reinterpret_cast<const long long*>(a->input_token);
  p.embed = static_cast<const __nv_bfloat16*>(a->embed_weights);
  p.out_token = reinterpret_cast<long long*>(a->output_token);
  p.lm_count = a->lm_head_instructions;
  if (++ctx->epoch == 0) ctx->epoch = 1;
  if (p.out_token && (ctx->epoch & 0xffffu) == 0) {
    // the argmax key carries the epoch's low 16 bits: restart it at the wrap
    cudaError_t e = cudaMemsetAsync(&ctx->status->argmax_key, 0, sizeof(unsigned long long),
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(argmax key)");
    ++ctx->epoch;
  }
  p.epoch = ctx->epoch;

  cudaError_t e = ek::launch_decode(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
  return EK_SUCCESS;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot call cudaMalloc at decode time: allocators that must not
// be re-entered, embedded runtimes that reserve all device memory up front and
// hand out only their own pool. For them the
// engine's scratch (status record, split-sum arrival counters, split partial
// sums) lives in file-scope device arrays of fixed size that every GPU which
// loads this library keeps until the process exits (about 0.7 MiB per GPU).
namespace {

constexpr size_t kStaticCounters = 65536;   // u32: L * 2 * (H / 16), e.g. L=64, H=8192
constexpr size_t kStaticPartials = 196608;  // bf16: (H / o_split + I / d_split) * H
constexpr int kMaxDevices = 64;

static __device__ __align__(256) ek::DevStatus g_static_status;
static __device__ __align__(256) unsigned g_static_counters[kStaticCounters];
static __device__ __align__(256) __nv_bfloat16 g_static_partials[kStaticPartials];

struct StaticScratch {
  bool ready = false;
  ek::DevStatus* status = nullptr;
  unsigned* counters = nullptr;
  __nv_bfloat16* partials = nullptr;
  unsigned epoch = 0;
};

std::mutex g_static_mu;
StaticScratch g_static[kMaxDevices];

}  // namespace

extern "C" int ek_llama_decode_static(const EkLlamaArgs* a, void* stream, EkStatus* status_out) {
  if (!a) return fail(EK_E_INVALID, "NULL arguments");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(EK_E_UNSUPPORTED, "device %d beyond %d", dev, kMaxDevices);

  // sizes the context path would allocate; reject instead of allocating
  const int H = a->hidden, I = a->intermediate, L = a->num_layers;
  const int dR = a->down_reduction_size > 0 ? a->down_reduction_size : I;
  const int oR = a->oproj_reduction_size > 0 ? a->oproj_reduction_size : H;
  if (H <= 0 || I <= 0 || L <= 0 || dR <= 0 || oR <= 0)
    return fail(EK_E_INVALID, "bad model dims");
  const size_t nctr = (size_t)L * 2 * (H / 16);
  const size_t npart = (size_t)(H / oR + I / dR) * H;
  if (nctr > kStaticCounters || npart > kStaticPartials)
    return fail(EK_E_UNSUPPORTED,
                "model needs %zu counters / %zu partial sums; the allocation-free entry point "
                "holds at most %zu / %zu",
                nctr, npart, kStaticCounters, kStaticPartials);

  EkContext tmp;
  {
    std::lock_guard<std::mutex> lk(g_static_mu);
    StaticScratch& s = g_static[dev];
    if (!s.ready) {  // first call on this device: resolve the arrays' device addresses
      if ((e = cudaGetSymbolAddress((void**)&s.status, g_static_status)) != cudaSuccess)
        return cuda_fail(e, "cudaGetSymbolAddress(status)");
      if ((e = cudaGetSymbolAddress((void**)&s.counters, g_static_counters)) != cudaSuccess)
        return cuda_fail(e, "cudaGetSymbolAddress(counters)");
      if ((e = cudaGetSymbolAddress((void**)&s.partials, g_static_partials)) != cudaSuccess)
        return cuda_fail(e, "cudaGetSymbolAddress(partials)");
      s.ready = true;
    }
    tmp.device = dev;
    tmp.status = s.status;
    tmp.counters = s.counters;
    tmp.counters_cap = kStaticCounters;
    tmp.partials = s.partials;
    tmp.partials_cap = kStaticPartials;
    tmp.epoch = s.epoch;
    // the epoch tags every arrival counter with this call, so values left by
    // earlier calls are ignored; advance it here under the lock
    do { ++s.epoch; } while (s.epoch == 0 || (s.epoch & 0xffffu) == 0);  // see the argmax key tag
    tmp.epoch = s.epoch - 1;  // ek_llama_decode pre-increments to s.epoch
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the status record must start clear for this call
  if ((e = cudaMemsetAsync(tmp.status, 0, sizeof(ek::DevStatus), st)) != cudaSuccess)
    return cuda_fail(e, "cudaMemsetAsync(status)");
  const int rc = ek_llama_decode(&tmp, a, stream);
  if (rc) return rc;
  if (status_out &&
      (e = cudaMemcpyAsync(status_out, tmp.status, sizeof(EkStatus), cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(status_out)");
  return EK_SUCCESS;
}

extern "C" int ek_mixtral_decode(EkContext* ctx, const EkMixtralArgs* a, void* stream) {
  if (!ctx || !a) return fail(EK_E_INVALID, "NULL context or arguments");
  const void* required[] = {a->barriers, a->instructions, a->qkv_weights, a->attn_ln_weights, a->o_weights,
                            a->expert_gate_weights, a->expert_up_weights, a->expert_down_weights,
                            a->router_weights, a->ffn_ln_weights, a->lm_head_norm_weights, a->lm_head_weights,
                            a->k_cache, a->v_cache, a->rope_cos, a->rope_sin, a->hidden_states, a->q_post_rope,
                            a->attn_out, a->attn_lse_intermediates, a->attn_out_intermediates,
                            a->expert_silu_out, a->router_normed_hidden, a->logits};
  for (size_t i = 0; i < sizeof(required) / sizeof(required[0]); ++i) {
    if (!required[i]) return fail(EK_E_INVALID, "pointer argument %zu is NULL", i);
    if (!aligned16(required[i])) return fail(EK_E_INVALID, "pointer argument %zu is not 16-byte aligned", i);
  }
  if (!a->selected_expert_indices || !a->selected_expert_scores || !a->predicted_expert_indices)
    return fail(EK_E_INVALID, "router output pointers must not be NULL");
  if (a->timings && !aligned16(a->timings)) return fail(EK_E_INVALID, "timings is not 16-byte aligned");
  const int L = a->num_layers, H = a->hidden, I = a->intermediate, D = a->head_dim;
  const int Hq = a->num_q_heads, Hkv = a->num_kv_heads, V = a->vocab, E = a->num_experts, K = a->experts_per_token;
  if (L < 1 || H < 256 || I < 256 || V < 16 || Hq < 1 || Hkv < 1)
    return fail(EK_E_INVALID, "bad model dims L=%d H=%d I=%d V=%d Hq=%d Hkv=%d", L, H, I, V, Hq, Hkv);
  if (E < 1 || E > ek::MAX_EXPERTS || K < 1 || K > ek::MAX_TOPK || K > E)
    return fail(EK_E_UNSUPPORTED, "experts %d / per token %d (max %d / %d)", E, K, ek::MAX_EXPERTS, ek::MAX_TOPK);
  if (D != 64 && D != 128) return fail(EK_E_UNSUPPORTED, "head_dim %d (supported: 64, 128)", D);
  if (H % 256 || I % 256) return fail(EK_E_INVALID, "hidden and intermediate must be multiples of 256");
  if (V % 16) return fail(EK_E_INVALID, "vocab %d not a multiple of 16", V);
  const bool tp = ctx->tp_connected && ctx->tp_world > 1;
  if (Hq % Hkv) return fail(EK_E_INVALID, "num_q_heads %% num_kv_heads != 0");
  if (!tp && Hq * D != H) return fail(EK_E_INVALID, "num_q_heads * head_dim must equal hidden");
  if ((Hq * D) % 256) return fail(EK_E_INVALID, "num_q_heads * head_dim must be a multiple of 256");
  if (tp) {
    if (L != ctx->tp_layers || H != ctx->tp_hidden || K != ctx->tp_topk || V * ctx->tp_world != ctx->tp_vocab)
      return fail(EK_E_INVALID, "dims differ from ek_tp_setup");
    if (a->logits != ctx->tp_buf + ctx->off_logits)
      return fail(EK_E_INVALID, "with tensor parallelism, logits must be the context's symmetric buffer");
    if (a->tp_lm_instructions < 0) return fail(EK_E_INVALID, "tp_lm_instructions < 0");
  }
  const int gqa = Hq / Hkv;
  if (gqa > ek::MAX_GQA || ek::CW * gqa * (D + 2) * 4 > ek::ACT_BYTES)
    return fail(EK_E_UNSUPPORTED, "GQA ratio %d too large for head_dim %d", gqa, D);
  if (I * 2 > ek::ACT_BYTES - 64 * 64) return fail(EK_E_UNSUPPORTED, "intermediate %d too large", I);
  if (a->kv_len < 1 || a->rope_rows < 1 || a->max_partials < 1)
    return fail(EK_E_INVALID, "kv_len, rope_rows and max_partials must be positive");
  if (a->pos_id < 0 || a->pos_id >= a->kv_len || a->pos_id >= a->rope_rows)
    return fail(EK_E_INVALID, "pos_id %d outside the KV cache or rope table", a->pos_id);
  if (a->barrier_rows < 8 || a->barrier_cols < Hq + 2 * Hkv || a->barrier_cols < E)
    return fail(EK_E_INVALID, "barriers must be at least [L, 8, max(Hq + 2 Hkv, E)]");
  if (a->queue_len < 1 || a->num_queues < 1) return fail(EK_E_INVALID, "empty instruction tensor");
  DeviceGuard g(ctx->device);
  int nsm = 0;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, ctx->device);
  if (a->num_queues > nsm) return fail(EK_E_INVALID, "%d instruction queues but only %d SMs", a->num_queues, nsm);
  int rc = grow(ctx, 1, 1);
  if (rc) return rc;

  KParams p;  // per call (thread-safe)
  std::memset(&p, 0, sizeof(p));
  const int qkv_rows = (Hq + 2 * Hkv) * D;
  const int tk = ek::HALF_STAGE / (D * 2);
  if ((rc = encode_kv(&p.tm_k, a->k_cache, (long long)L * a->kv_len, Hkv, D, tk, "k_cache"))) return rc;
  if ((rc = encode_kv(&p.tm_v, a->v_cache, (long long)L * a->kv_len, Hkv, D, tk, "v_cache"))) return rc;
  p.w_qkv = static_cast<const __nv_bfloat16*>(a->qkv_weights);
  p.w_o = static_cast<const __nv_bfloat16*>(a->o_weights);
  p.w_lm = static_cast<const __nv_bfloat16*>(a->lm_head_weights);
  p.w_egate = static_cast<const __nv_bfloat16*>(a->expert_gate_weights);
  p.w_eup = static_cast<const __nv_bfloat16*>(a->expert_up_weights);
  p.w_edown = static_cast<const __nv_bfloat16*>(a->expert_down_weights);
  p.w_router = static_cast<const __nv_bfloat16*>(a->router_weights);
  p.ffn_ln = static_cast<const __nv_bfloat16*>(a->ffn_ln_weights);
  p.rows_qkv = (long long)L * qkv_rows;
  p.rows_o = (long long)L * H;
  p.rows_lm = V;
  p.rows_eup = (long long)L * E * I;
  p.rows_edown = (long long)L * E * H;
  p.barriers = a->barriers;
  p.instructions = a->instructions;
  p.timings = a->timings;
  p.attn_ln = static_cast<const __nv_bfloat16*>(a->attn_ln_weights);
  p.lm_norm = static_cast<const __nv_bfloat16*>(a->lm_head_norm_weights);
  p.k_cache = static_cast<__nv_bfloat16*>(a->k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(a->v_cache);
  p.rope_cos = a->rope_cos;
  p.rope_sin = a->rope_sin;
  p.hidden = static_cast<__nv_bfloat16*>(a->hidden_states);
  p.q = static_cast<__nv_bfloat16*>(a->q_post_rope);
  p.attn_out = static_cast<__nv_bfloat16*>(a->attn_out);
  p.lse = a->attn_lse_intermediates;
  p.attn_o = a->attn_out_intermediates;
  p.expert_silu = static_cast<__nv_bfloat16*>(a->expert_silu_out);
  p.router_normed = static_cast<__nv_bfloat16*>(a->router_normed_hidden);
  p.logits = static_cast<__nv_bfloat16*>(a->logits);
  p.sel_idx = a->selected_expert_indices;
  p.sel_scores = static_cast<__nv_bfloat16*>(a->selected_expert_scores);
  p.pred_idx = a->predicted_expert_indices;
  p.status = ctx->status;
  p.split_counters = ctx->counters;
  p.split_partials = ctx->partials;
  p.model = ek::MODEL_MIXTRAL;
  p.E = E;
  p.topk = K;
  p.down_done_target = K * (H / 16);
  p.L = L; p.H = H; p.I = I; p.D = D; p.Hq = Hq; p.Hkv = Hkv; p.V = V;
  p.T = a->kv_len; p.rope_rows = a->rope_rows; p.maxP = a->max_partials;
  p.brow = a->barrier_rows; p.bcol = a->barrier_cols;
  p.nq = a->num_queues; p.Q = a->queue_len;
  p.qkv_rows = qkv_rows; p.gqa = gqa; p.tk = tk;
  p.pos = a->pos_id; p.skip_red = a->skip_attn_reduction ? 1 : 0;
  p.scale = a->attn_scale; p.eps = a->rms_norm_eps;
  p.down_R = I; p.o_R = Hq * D; p.down_splits = 1; p.o_splits = 1;
  p.tp_world = 1;
  p.spec_stages = a->speculative_prefetch_stages > 0 ? a->speculative_prefetch_stages : 0;
  if (tp) {
    p.tp_world = ctx->tp_world;
    p.tp_rank = ctx->tp_rank;
    for (int r = 0; r < ctx->tp_world; ++r) p.tp_peer[r] = ctx->tp_peer[r];
    p.tp_off_recv_o = ctx->off_recv_o;
    p.tp_off_recv_d = ctx->off_recv_d;
    p.tp_off_cnt_o = ctx->off_cnt_o;
    p.tp_off_cnt_d = ctx->off_cnt_d;
    p.tp_off_cnt_lm = ctx->off_cnt_lm;
    p.tp_off_logits = ctx->off_logits;
    p.lm_row0 = ctx->tp_rank * V;
    p.tp_lm_count = a->tp_lm_instructions;
    p.tp_step = ++ctx->tp_step;
  }
  p.pf_stages = a->l2_prefetch_stages > 0 ? a->l2_prefetch_stages : 0;
  p.pf_next = a->l2_prefetch_stages < 0 ? min(-a->l2_prefetch_stages, 2) : 0;
  p.pf_mlp = a->cache_flags;
  p.pf_gap_ns = a->prefetch_gap_ns > 0 ? (unsigned)a->prefetch_gap_ns : 0u;
  p.record = a->record_timings && a->timings ? 1 : 0;
  p.timeout_ns = a->timeout_ns > 0 ? a->timeout_ns : 1000000000ll;
  if (++ctx->epoch == 0) ctx->epoch = 1;
  p.epoch = ctx->epoch;
  cudaError_t e = ek::launch_decode(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
  return EK_SUCCESS;
}
