// Persistent batch-1 decode megakernel for B200 (sm_100a).
//
// One thread block per SM. Block b interprets instruction queue b
// (instructions[b, i, 0..31], the words of megakernels/instructions.py
// `Instruction.serialize`). The block has two roles:
//
//   loader   (warp CW, one lane) walks the queue ahead of the consumers and
//            streams every weight tile and every *past* KV-cache tile that
//            the queue will read into a ring of 16 KiB shared-memory stages
//            with TMA (cp.async.bulk.tensor). Optionally it also issues
//            cp.async.bulk.prefetch.tensor into L2 for stages beyond the
//            ring. None of that data depends on other SMs, so the loader
//            never waits on a cross-SM counter. It stalls only when the ring
//            is full, and it keeps HBM busy while the consumers wait.
//   consumers (warps 0..CW-1) execute the instructions in order: wait for the
//            producer counters (bounded spin on `barriers`), stage the
//            activation vector (RMSNorm'd hidden, attn_out, silu_out) in
//            shared memory, then reduce the ring stages with vectorised bf16
//            loads, fp32 FMA and warp shuffles. The epilogue writes results
//            and bumps counters.
//
// Rounding follows the reference PyTorch interpreter step by step
// (megakernels/demos/latency/python_vm.py): matvec outputs are rounded to bf16
// before RoPE, SiLU or the residual add, RMSNorm rounds x * rsqrt(var + eps)
// to bf16 before the weight multiply, and attention runs in fp32. Column-split
// residual adds (DownProjResidual) are applied in split order by the last
// split to arrive, so the result is deterministic.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#include "ek_ptx.cuh"

// Compile-time variant of the translation unit that includes this header
// (ek_decode.cu is compiled once per variant, so that each kernel carries only
// the code its model runs: a megakernel's code must stay small enough for the
// SM's instruction cache).
//   EK_MODEL 0: Llama opcodes 1-7; 1: Mixtral opcodes 1-8 (and tensor parallel)
//   EK_PF    0: no L2 prefetch paths; 1: the optional L2 prefetch modes
#ifndef EK_MODEL
#define EK_MODEL 0
#endif
#ifndef EK_PF
#define EK_PF 0
#endif

namespace ek {

constexpr bool kMixtral = EK_MODEL == 1;
constexpr bool kPrefetch = EK_PF == 1;

constexpr int CW = 8;                 // consumer warps
constexpr int NC = CW * 32;           // consumer threads
constexpr int LOADER_WARP = CW;       // warp index of the ring loader
constexpr int PREFETCH_WARP = CW + 1; // warp index of the MLP-weight L2 prefetcher (prefetch variant)
constexpr int NTHREADS = NC + (kPrefetch ? 64 : 32);  // + loader warp (+ prefetcher warp)
constexpr int STAGE_BYTES = 16384;    // one ring stage
constexpr int HALF_STAGE = 8192;      // one TMA box (16 rows x 256 bf16, or TK x D bf16)
constexpr int ACT_BYTES = 49152;      // activation vector + per-stage partial sums / attention merge
// Ring slots. Every consumer warp reads every stage in stream order (the
// GEMVs split a stage's pieces over all warps), so a warp waiting on a slot is
// never more than one lap ahead of it and any slot count works. 8 slots keep
// the shared-memory carve-out small enough to leave L1 for the threads' stacks.
#ifndef EK_STAGES
#define EK_STAGES 8
#endif
constexpr int NUM_STAGES = EK_STAGES;  // 8: 128 KiB ring
constexpr int CTRL_BYTES = 1024;      // mbarriers + reduction scratch
constexpr int SMEM_BYTES = NUM_STAGES * STAGE_BYTES + ACT_BYTES + CTRL_BYTES;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
constexpr int MAX_GQA = 4;  // query heads per KV head
constexpr int MAX_EXPERTS = 16;
constexpr int MAX_TOPK = 4;
constexpr int LM_HEAD_SPLIT = 2048;
constexpr int MAX_TP = 8;  // most tensor-parallel ranks (symmetric buffers mapped per launch)

enum Op : int {
  OP_NOOP = 0,
  OP_QKV = 1,
  OP_PARTIAL = 2,
  OP_REDUCTION = 3,
  OP_OPROJ = 4,
  OP_UPGATE = 5,
  OP_DOWN = 6,
  OP_LM_HEAD = 7,
  OP_PREDICT = 8,  // Mixtral SpeculativeExpertPredict
};

// Slots of timings[queue][instruction][128] (globaltimer ns, low 31 bits),
// following the reference's TEVENT convention (include/util.cuh:221-245 of
// epic-kernel) so that its timing plots read them.
constexpr int TS_START = 0;        // TEVENT_CONTROLLER_START: instruction begins
constexpr int TS_END = 4;          // TEVENT_CONTROLLER_END: instruction done
constexpr int TS_WAIT = 44;        // TEVENT_AT_GMEM_WAIT: counter wait begins
constexpr int TS_READY = 45;       // TEVENT_DONE_GMEM_WAIT: dependencies satisfied
constexpr int TS_STORE = 46;       // TEVENT_AT_GMEM_STORE: epilogue (results, counters) begins
constexpr int TS_FIRST_USE = 49;   // TEVENT_FIRST_USE: first ring stage acquired
constexpr int TS_LAST_USE = 52;    // TEVENT_LAST_USE: last ring stage consumed
constexpr int TS_ACT = 55;         // activation vector staged in shared memory (free slot)
constexpr int TS_STAGE_USE = 56;   // + k (k < 28): consumers acquired ring stage k
constexpr int TS_STAGE_LOAD = 84;  // + k (k < 16): loader issued ring stage k
constexpr int TS_PREFETCH = 100;   // 100 / 101: MLP prefetcher start / end (prefetch variant)
constexpr int TS_DIAG = 126;       // instruction 0 only: 126 prefetched stages, 127 loaded stages

enum CacheBits : int {
  PF_UPGATE = 1,
  PF_DOWN = 2,
  PF_BULK = 4,
  PF_EVICT_LAST = 8,
  PF_RING_EVICT_FIRST = 16,
  PF_KV_EVICT_FIRST = 32,
};

enum Model : int { MODEL_LLAMA = 0, MODEL_MIXTRAL = 1 };

// Device status record; layout of EkStatus followed by the abort word.
struct DevStatus {
  int code, sm, instr, opcode, layer, observed, expected, detail;
  unsigned abort_epoch;  // == current epoch once any block failed in this launch
  int pad0;
  // fused argmax of the logits (Llama, output_token set): the best
  // (epoch16, ordered bf16 value, ~row) key of the launch, and the LM-head
  // instructions finished per launch in a ring of 4 counters (slot epoch % 4;
  // block 0 clears the next launch's slot when it starts)
  unsigned long long argmax_key;
  unsigned lm_arrivals[4];
};
static_assert(sizeof(DevStatus) == 64, "status record");

struct KParams {
  CUtensorMap tm_k, tm_v;  // KV caches [L*T, Hkv, D], box D x 1 x tk

  const __nv_bfloat16* w_qkv;  // [L * qkv_rows, H]
  const __nv_bfloat16* w_o;    // [L * H, Hq * D]
  const __nv_bfloat16* w_up;   // [L * I, H]
  const __nv_bfloat16* w_gate; // [L * I, H]
  const __nv_bfloat16* w_down; // [L * H, I]
  const __nv_bfloat16* w_lm;   // [V, H]
  long long rows_qkv, rows_o, rows_up, rows_down, rows_lm;  // matrix rows (bounds checks)

  // Mixtral (model == MODEL_MIXTRAL); opcodes 5/6/7 change meaning, 8 is added
  const __nv_bfloat16* w_egate;   // [L * E * I, H]
  const __nv_bfloat16* w_eup;     // [L * E * I, H]
  const __nv_bfloat16* w_edown;   // [L * E * H, I]
  const __nv_bfloat16* w_router;  // [L * E, H]
  const __nv_bfloat16* ffn_ln;    // [L, H]
  __nv_bfloat16* expert_silu;     // [E, I]
  __nv_bfloat16* router_normed;   // [H]
  int* sel_idx;                   // [topk]
  __nv_bfloat16* sel_scores;      // [topk]
  int* pred_idx;                  // [topk]
  long long rows_eup, rows_edown;

  // Mixtral tensor parallelism (tp_world > 1): symmetric buffers of all ranks
  int tp_world, tp_rank;
  unsigned tp_step;          // launches since ek_tp_connect (counters are cumulative)
  char* tp_peer[8];          // base of each rank's symmetric buffer (tp_peer[tp_rank] = own)
  long long tp_off_recv_o, tp_off_recv_d, tp_off_cnt_o, tp_off_cnt_d, tp_off_cnt_lm, tp_off_logits;
  int lm_row0;               // first global vocabulary row of this rank's LM-head shard
  int tp_lm_count;           // LM-head instructions per rank and launch

  int* barriers;
  const int* instructions;
  int* timings;
  const __nv_bfloat16* attn_ln;
  const __nv_bfloat16* mlp_ln;
  const __nv_bfloat16* lm_norm;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  const float* rope_cos;
  const float* rope_sin;
  __nv_bfloat16* hidden;
  __nv_bfloat16* q;
  __nv_bfloat16* attn_out;
  float* lse;
  float* attn_o;
  __nv_bfloat16* silu;
  __nv_bfloat16* logits;
  DevStatus* status;
  unsigned* split_counters;       // [L][2][H/16] epoch-tagged arrival counters
  __nv_bfloat16* split_partials;  // [2][max_splits][H] bf16 partial sums

  int model, E, topk;
  int down_done_target;  // counter value of a finished layer (Llama: splits * H/16, Mixtral: k * H/16)
  int L, H, I, D, Hq, Hkv, V, T, rope_rows, maxP, brow, bcol, nq, Q;
  int qkv_rows, gqa, tk;
  int pos, skip_red;
  float scale, eps;
  int down_R, o_R, down_splits, o_splits;
  int pf_stages, record;
  // L2 prefetch at instruction granularity (off by default: both measured
  // slower): 1 = the next instruction's weights when an instruction starts
  // loading; 2 = this queue's up/gate and down weights of a layer when its
  // first attention-chain instruction (opcodes 1-4) starts loading.
  int pf_next;
  // EK_CACHE_* bits (include/ek.h). Prefetch bits (prefetch variant only):
  // L2 prefetch of a layer's MLP weights by the prefetcher warp, issued once
  // the previous layer's down projection is complete.
  int pf_mlp;
  unsigned pf_gap_ns;  // pause of the prefetcher warp after each 16 KiB it requests
  // Llama with column-split down projections (and one O-proj split): layers
  // l < defer_down publish only their bf16 split partials; the next readers
  // of the residual stream (layer l + 1's QKV RMSNorm and O-proj residual add)
  // add them to `hidden` in split order, the interpreter's order and rounding.
  // The last layer of the instruction stream adds them itself, so the LM head
  // and the caller see the final hidden state.
  int defer_down;
  // The last PartialAttention of a KV head to finish runs that head's
  // AttentionReduction; the reduction instructions become no-ops. Only for
  // schedules whose reductions are terminal over all partials in order.
  int fuse_red;
  // fused embedding gather and argmax (Llama): layer 0 reads the residual
  // stream from embed[*in_token] instead of `hidden`; the LM head writes the
  // first index of the largest logit to *out_token once all lm_count LM-head
  // instructions finished
  const long long* in_token;
  const __nv_bfloat16* embed;
  long long* out_token;
  int lm_count;
  int spec_stages;  // Mixtral: stages per predicted expert L2-prefetched before the router handoff
  long long timeout_ns;
  unsigned epoch;
};

// ------------------------------------------------------------------ decoding
struct Ins {
  int w[32];
};

__device__ __forceinline__ void fetch_ins(const KParams& p, int q, int i, Ins& ins) {
  const int4* src = reinterpret_cast<const int4*>(p.instructions + ((size_t)q * p.Q + i) * 32);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    int4 v = __ldg(src + k);
    ins.w[4 * k + 0] = v.x;
    ins.w[4 * k + 1] = v.y;
    ins.w[4 * k + 2] = v.z;
    ins.w[4 * k + 3] = v.w;
  }
}

// A GEMV ring stage holds `rps` row segments of up to 8192 bf16 (16 KiB)
// streamed by 1-D bulk copies: 4 rows of 2048, 2 rows of 3072 or 4096, 8 rows
// of 1024, 16 rows of 512, or, for segments longer than 8192, one row in
// `chunks` column chunks (8192 + 6144 for 14336). Segment = the columns of a row
// an instruction reduces over.
struct GemvShape {
  int rps;     // rows per stage (1, 2, 4, 8 or 16)
  int chunks;  // stages per row segment
};

__device__ __forceinline__ GemvShape gemv_shape(int S) {
  GemvShape g;
  if (S > STAGE_BYTES / 2) {
    g.rps = 1;
    g.chunks = (S + STAGE_BYTES / 2 - 1) / (STAGE_BYTES / 2);
  } else {
    const int r = (STAGE_BYTES / 2) / S;
    g.rps = r >= 16 ? 16 : r >= 8 ? 8 : r >= 4 ? 4 : r >= 2 ? 2 : 1;
    g.chunks = 1;
  }
  return g;
}

// Ring stages per 16-row block for a row segment of S columns.
__device__ __forceinline__ int stages_per_row_block(int S) {
  const GemvShape g = gemv_shape(S);
  return (16 / g.rps) * g.chunks;
}

// Floats of partial row sums one 16-row GEMV block leaves: 16 rows x CW warps.
constexpr int BLOCK_PART = 16 * CW;

// Bytes of `act` a GEMV instruction needs: its activation slice (K bf16) and
// the partial sums of its ns ring stages of S-column row segments.
__device__ __forceinline__ int gemv_act_bytes(int K, int ns, int S = -1) {
  return ((K * 2 + 15) & ~15) + (ns / stages_per_row_block(S < 0 ? K : S)) * BLOCK_PART * 4;
}

// Token range [t_begin, t_end) of one partial (python_vm.py:306-318), and the
// end of the part the loader may stream (tokens before pos_id).
struct TokenRange {
  int t_begin, t_end, t_load_end;
};

__device__ __forceinline__ TokenRange partial_tokens(const KParams& p, int num_partials, int partial) {
  const int seq = p.pos + 1;
  const int total_blocks = (seq + 15) / 16;
  const int per_partial = (total_blocks + num_partials - 1) / num_partials;
  const int b0 = partial * per_partial;
  const int b1 = min(b0 + per_partial, total_blocks);
  TokenRange r;
  r.t_begin = b0 * 16;
  r.t_end = min(b1 * 16, seq);
  if (r.t_end < r.t_begin) r.t_end = r.t_begin;
  r.t_load_end = max(r.t_begin, min(r.t_end, p.pos));
  return r;
}

// What an instruction streams through the ring. Loader and consumers call the
// same function, so both agree on the number of stages.
struct Plan {
  int op;
  int layer;
  int ns;         // ring stages
  int bad_word;   // >= 0: index of an out-of-range word
};

__device__ __forceinline__ Plan make_plan(const KParams& p, const Ins& ins) {
  Plan pl;
  pl.op = ins.w[0];
  pl.layer = 0;
  pl.ns = 0;
  pl.bad_word = -1;
  const int* w = ins.w;
  auto bad = [&](int idx) {
    pl.bad_word = idx;
    pl.ns = 0;
  };
  if (kMixtral && pl.op >= OP_UPGATE && pl.op <= OP_PREDICT) {
    switch (pl.op) {
      case OP_UPGATE: {  // RmsRouterUpgate: layer, start_block, num_blocks
        pl.layer = w[1];
        if (w[1] < 0 || w[1] >= p.L) { bad(1); break; }
        if (w[2] < 0) { bad(2); break; }
        if (w[3] < 0 || w[2] + w[3] > p.I / 16) { bad(3); break; }
        pl.ns = p.topk * w[3] * 2 * stages_per_row_block(p.H);
        if (gemv_act_bytes(p.H, pl.ns) > ACT_BYTES) { bad(3); break; }
        break;
      }
      case OP_DOWN: {  // ExpertDownProjFused: layer, start_block, end_block, 0
        pl.layer = w[1];
        if (w[1] < 0 || w[1] >= p.L) { bad(1); break; }
        if (w[2] < 0 || w[2] > w[3]) { bad(2); break; }
        if (w[3] > p.H / 16) { bad(3); break; }
        if (w[4] != 0) { bad(4); break; }
        pl.ns = p.topk * (w[3] - w[2]) * stages_per_row_block(p.I);
        if (gemv_act_bytes(p.I, pl.ns) > ACT_BYTES) { bad(3); break; }
        break;
      }
      case OP_LM_HEAD: {  // Mixtral_RMS_LM_Head: start_block, end_block, split
        pl.layer = p.L - 1;
        if (w[1] < 0 || w[1] > w[2]) { bad(1); break; }
        if (w[2] > p.V / 16) { bad(2); break; }
        if (w[3] < 0 || (w[3] + 1) * LM_HEAD_SPLIT > p.H) { bad(3); break; }
        pl.ns = (w[2] - w[1]) * stages_per_row_block(LM_HEAD_SPLIT);
        if (gemv_act_bytes(p.H, pl.ns, LM_HEAD_SPLIT) > ACT_BYTES) { bad(2); break; }
        break;
      }
      case OP_PREDICT: {  // SpeculativeExpertPredict: layer
        pl.layer = w[1];
        if (w[1] < 0 || w[1] >= p.L) bad(1);
        break;
      }
    }
    return pl;
  }
  switch (pl.op) {
    case OP_NOOP:
      break;
    case OP_QKV: {
      pl.layer = w[1];
      if (w[1] < 0 || w[1] >= p.L) { bad(1); break; }
      if (w[2] < 0 || w[2] > w[3]) { bad(2); break; }
      if (w[3] > p.qkv_rows / 16) { bad(3); break; }
      pl.ns = (w[3] - w[2]) * stages_per_row_block(p.H);
      if (gemv_act_bytes(p.H, pl.ns) > ACT_BYTES) { bad(3); break; }
      break;
    }
    case OP_PARTIAL: {
      pl.layer = w[1];
      if (w[1] < 0 || w[1] >= p.L) { bad(1); break; }
      if (w[2] < 0 || w[2] >= p.Hkv) { bad(2); break; }
      if (w[3] < 1) { bad(3); break; }
      if (w[4] < 0 || w[4] >= w[3] || w[4] >= p.maxP) { bad(4); break; }
      if (p.pos < 0 || p.pos >= p.T || p.pos >= p.rope_rows) { bad(0); break; }
      TokenRange r = partial_tokens(p, w[3], w[4]);
      pl.ns = (r.t_load_end - r.t_begin + p.tk - 1) / p.tk;
      break;
    }
    case OP_REDUCTION: {
      pl.layer = w[1];
      if (w[1] < 0 || w[1] >= p.L) { bad(1); break; }
      if (w[2] < 0 || w[2] + p.gqa > p.Hq) { bad(2); break; }
      if (w[5] < 1 || w[5] > 25) { bad(5); break; }
      for (int j = 0; j < w[5]; ++j)
        if (w[6 + j] < 0 || w[6 + j] >= p.maxP) { bad(6 + j); break; }
      if (pl.bad_word >= 0) break;
      if (!w[4] && (w[6 + w[5]] < 0 || w[6 + w[5]] >= p.maxP)) { bad(6 + w[5]); break; }
      break;
    }
    case OP_OPROJ:
    case OP_DOWN: {
      pl.layer = w[1];
      const int R = pl.op == OP_OPROJ ? p.o_R : p.down_R;
      const int splits = pl.op == OP_OPROJ ? p.o_splits : p.down_splits;
      if (w[1] < 0 || w[1] >= p.L) { bad(1); break; }
      if (w[2] < 0 || w[2] > w[3]) { bad(2); break; }
      if (w[3] > p.H / 16) { bad(3); break; }
      if (w[4] < 0 || w[4] >= splits) { bad(4); break; }
      pl.ns = (w[3] - w[2]) * stages_per_row_block(R);
      if (gemv_act_bytes(R, pl.ns) > ACT_BYTES) { bad(3); break; }
      break;
    }
    case OP_UPGATE: {
      pl.layer = w[1];
      if (w[1] < 0 || w[1] >= p.L) { bad(1); break; }
      if (w[2] < 0 || w[2] > 29) { bad(2); break; }
      for (int j = 0; j < w[2]; ++j)
        if (w[3 + j] < 0 || w[3 + j] >= p.I / 16) { bad(3 + j); break; }
      if (pl.bad_word >= 0) break;
      pl.ns = w[2] * 2 * stages_per_row_block(p.H);
      if (gemv_act_bytes(p.H, pl.ns) > ACT_BYTES) { bad(2); break; }
      break;
    }
    case OP_LM_HEAD: {
      pl.layer = p.L - 1;
      if (w[1] < 0 || w[1] > w[2]) { bad(1); break; }
      if (w[2] > p.V / 16) { bad(2); break; }
      pl.ns = (w[2] - w[1]) * stages_per_row_block(p.H);
      if (gemv_act_bytes(p.H, pl.ns) > ACT_BYTES) { bad(2); break; }
      break;
    }
    default:
      pl.bad_word = 0;
      break;
  }
  return pl;
}

// Coordinates of ring stage k of an instruction. `issue` decides between the
// TMA load into shared memory and the L2 prefetch.
// ------------------------------------------------------------------ errors
__device__ __forceinline__ bool aborted(const KParams& p) {
  return ld_relaxed(reinterpret_cast<const int*>(&p.status->abort_epoch)) == (int)p.epoch;
}

static __device__ __noinline__ void record_error(const KParams& p, int code, int instr, int opcode, int layer,
                             int observed, int expected, int detail) {
  if (atomicCAS(&p.status->code, 0, -1) == 0) {
    p.status->sm = blockIdx.x;
    p.status->instr = instr;
    p.status->opcode = opcode;
    p.status->layer = layer;
    p.status->observed = observed;
    p.status->expected = expected;
    p.status->detail = detail;
    __threadfence();
    atomicExch(&p.status->code, code);
  }
  atomicExch(&p.status->abort_epoch, p.epoch);
}

// Loader-side walk over an instruction's ring stages, in the order the
// consumers number them (column chunk fastest, then row group, matrix
// (up, gate), block). Advancing costs a few additions; the per-instruction
// set-up does the divisions once.
struct StageWalker {
  int op, k, ns;
  // GEMV
  const __nv_bfloat16* mat[2];
  long long mat_rows;
  const int* w;
  int nmat, stride, col0, S, rps, chunks, groups;  // groups = 16 / rps
  int j, m, rg, c;
  long long row_base;  // first matrix row of block j
  int es, ne;                 // expert slot (Mixtral expert ops), slots
  int experts[MAX_TOPK];
  int nblocks;
  // attention
  int kv_t0, kv_head;

  __device__ __forceinline__ long long block_row(const KParams& p, int jj) const {
    if (kMixtral) {
      const long long e = (long long)w[1] * p.E + experts[es];
      switch (op) {
        case OP_UPGATE: return e * p.I + (long long)(w[2] + jj) * 16;
        case OP_DOWN: return e * p.H + (long long)(w[2] + jj) * 16;
        case OP_LM_HEAD: return (long long)(w[1] + jj) * 16;
        default: break;
      }
    }
    switch (op) {
      case OP_QKV: return (long long)w[1] * p.qkv_rows + (long long)(w[2] + jj) * 16;
      case OP_OPROJ:
      case OP_DOWN: return (long long)w[1] * p.H + (long long)(w[2] + jj) * 16;
      case OP_UPGATE: return (long long)w[1] * p.I + (long long)w[3 + jj] * 16;
      default: return (long long)(w[1] + jj) * 16;  // OP_LM_HEAD
    }
  }

  // `ex`: the selected (or, for prefetch, predicted) experts of a Mixtral
  // expert instruction; ignored otherwise.
  __device__ __forceinline__ void init(const KParams& p, const Ins& ins, const Plan& pl, const int* ex = nullptr) {
    op = pl.op;
    k = 0;
    ns = pl.ns;
    w = ins.w;
    nmat = 1;
    col0 = 0;
    es = 0;
    ne = 1;
    nblocks = 1 << 30;
    if (kMixtral && (op == OP_UPGATE || op == OP_DOWN || op == OP_LM_HEAD)) {
      if (op == OP_UPGATE) {
        mat[0] = p.w_egate; mat[1] = p.w_eup; nmat = 2; mat_rows = p.rows_eup;
        stride = p.H; S = p.H; nblocks = w[3]; ne = p.topk;
      } else if (op == OP_DOWN) {
        mat[0] = p.w_edown; mat_rows = p.rows_edown; stride = p.I; S = p.I;
        nblocks = w[3] - w[2]; ne = p.topk;
      } else {
        mat[0] = p.w_lm; mat_rows = p.rows_lm; stride = p.H; S = LM_HEAD_SPLIT; col0 = w[3] * LM_HEAD_SPLIT;
      }
      for (int i = 0; i < MAX_TOPK; ++i) {
        int e = ex ? ex[i < p.topk ? i : 0] : 0;
        experts[i] = (e < 0 || e >= p.E) ? 0 : e;
      }
      const GemvShape g = gemv_shape(S);
      rps = g.rps;
      chunks = g.chunks;
      groups = 16 / rps;
      j = m = rg = c = 0;
      if (ns > 0) row_base = block_row(p, 0);
      return;
    }
    switch (op) {
      case OP_QKV: mat[0] = p.w_qkv; mat_rows = p.rows_qkv; stride = p.H; S = p.H; break;
      case OP_OPROJ: mat[0] = p.w_o; mat_rows = p.rows_o; stride = p.Hq * p.D; S = p.o_R; col0 = w[4] * p.o_R; break;
      case OP_DOWN: mat[0] = p.w_down; mat_rows = p.rows_down; stride = p.I; S = p.down_R; col0 = w[4] * p.down_R; break;
      case OP_UPGATE: mat[0] = p.w_up; mat[1] = p.w_gate; mat_rows = p.rows_up; nmat = 2; stride = p.H; S = p.H; break;
      case OP_LM_HEAD: mat[0] = p.w_lm; mat_rows = p.rows_lm; stride = p.H; S = p.H; break;
      case OP_PARTIAL: {
        const TokenRange r = partial_tokens(p, w[3], w[4]);
        kv_t0 = w[1] * p.T + r.t_begin;
        kv_head = w[2];
        return;
      }
      default: return;
    }
    const GemvShape g = gemv_shape(S);
    rps = g.rps;
    chunks = g.chunks;
    groups = 16 / rps;
    j = m = rg = c = 0;
    if (ns > 0) row_base = block_row(p, 0);
  }

  __device__ __forceinline__ bool done() const { return k >= ns; }

  // Issue the current stage (load into dst completing on bar, or an L2
  // prefetch) and advance. Returns the stage's bytes.
  template <bool PREFETCH>
  __device__ __forceinline__ uint32_t issue(const KParams& p, uint8_t* dst, uint64_t* bar) {
    uint32_t bytes;
    if (op == OP_PARTIAL) {
      const int t0 = kv_t0 + k * p.tk;
      if (PREFETCH) {
        tma_prefetch_3d(&p.tm_k, 0, kv_head, t0);
        tma_prefetch_3d(&p.tm_v, 0, kv_head, t0);
      } else {
        mbar_arrive_expect_tx(bar, 2 * HALF_STAGE);
        if (p.pf_mlp & PF_KV_EVICT_FIRST) {
          const uint64_t pol = policy_evict_first();
          tma_load_3d_hint(dst, &p.tm_k, 0, kv_head, t0, bar, pol);
          tma_load_3d_hint(dst + HALF_STAGE, &p.tm_v, 0, kv_head, t0, bar, pol);
        } else {
          tma_load_3d(dst, &p.tm_k, 0, kv_head, t0, bar);
          tma_load_3d(dst + HALF_STAGE, &p.tm_v, 0, kv_head, t0, bar);
        }
      }
      bytes = 2 * HALF_STAGE;
    } else {
      const int col = col0 + c * (STAGE_BYTES / 2);
      const int len = min(STAGE_BYTES / 2, S - c * (STAGE_BYTES / 2));
      const uint32_t row_bytes = (uint32_t)len * 2;
      bytes = row_bytes * rps;
      const long long row = row_base + rg * rps;
      const __nv_bfloat16* src = mat[m] + row * stride + col;
      const bool whole = len == stride;  // consecutive whole rows: one copy
      // self-check: rows, columns, size and 16-byte alignment of the copy
      if (row < 0 || row + rps > mat_rows || col < 0 || col + len > stride || len <= 0 ||
          bytes > (uint32_t)STAGE_BYTES || ((reinterpret_cast<uintptr_t>(src) | row_bytes) & 15u)) {
        record_error(p, 5, k, op, (int)(row >> 32), (int)row, col, len);
        if (!PREFETCH) mbar_arrive_expect_tx(bar, 0);  // completes the phase, no copy
        advance(p);
        return 0;
      }
      if (PREFETCH) {
        if (whole) bulk_prefetch_l2(src, bytes);
        else for (int i = 0; i < rps; ++i) bulk_prefetch_l2(src + (size_t)i * stride, row_bytes);
      } else {
        mbar_arrive_expect_tx(bar, bytes);
        if (p.pf_mlp & PF_RING_EVICT_FIRST) {
          const uint64_t pol = policy_evict_first();
          if (whole) bulk_load_hint(dst, src, bytes, bar, pol);
          else for (int i = 0; i < rps; ++i) bulk_load_hint(dst + i * row_bytes, src + (size_t)i * stride, row_bytes, bar, pol);
        } else {
          if (whole) bulk_load(dst, src, bytes, bar);
          else for (int i = 0; i < rps; ++i) bulk_load(dst + i * row_bytes, src + (size_t)i * stride, row_bytes, bar);
        }
      }
    }
    advance(p);
    return bytes;
  }

  // Fast path: the number of stages from here on that follow each other at a
  // fixed stride in one matrix: a stage is `copies` copies of `bytes` each,
  // copy c at src + c * row_step, and the next stage starts stage_step bytes
  // further (one copy per stage for whole rows, one per row for row segments
  // of a column split). 0 if the current stage needs the general path. The
  // run's bounds and alignment are checked here, once.
  // A run of whole rows longer than a stage (chunks > 1; Mixtral's expert
  // down projection, 14336 columns) is contiguous too: its stages alternate
  // between full chunks of `bytes` and a last chunk of `last_bytes`, and the
  // source advances by each stage's size (chunk c0 first).
  struct Run {
    const uint8_t* src;
    uint32_t bytes, last_bytes;
    int copies, chunks, c0;
    long long row_step, stage_step;
  };
  __device__ __forceinline__ int contiguous_run(const KParams& p, Run& r) {
    if (op == OP_PARTIAL) return 0;
    r.chunks = chunks;
    r.c0 = c;
    if (chunks != 1) {
      if (S != stride || col0 != 0 || rps != 1 || nmat != 1) return 0;
      const long long per_expert = (long long)(nblocks < (1 << 29) ? nblocks : 0) * groups * chunks;
      const long long at = ((long long)j * groups + rg) * chunks + c;
      const int n = (int)min((long long)(ns - k), per_expert - at);
      const long long row = row_base + rg;
      r.copies = 1;
      r.bytes = STAGE_BYTES;
      r.last_bytes = (uint32_t)(S - (chunks - 1) * (STAGE_BYTES / 2)) * 2;
      r.row_step = r.stage_step = 0;
      r.src = reinterpret_cast<const uint8_t*>(mat[m] + row * stride + (long long)c * (STAGE_BYTES / 2));
      if (n < 1 || row < 0 || row + (c + n + chunks - 1) / chunks > mat_rows || r.last_bytes == 0 ||
          r.last_bytes > (uint32_t)STAGE_BYTES || ((reinterpret_cast<uintptr_t>(r.src) | r.last_bytes) & 15u))
        return 0;
      return n;
    }
    int n = groups - rg;
    if (nmat == 1) n = (int)min((long long)(ns - k), (long long)(nblocks - j) * groups - rg);
    const long long row = row_base + (long long)rg * rps;
    const bool whole = S == stride && col0 == 0;
    r.copies = whole ? 1 : rps;
    r.bytes = (uint32_t)(whole ? rps * S * 2 : S * 2);
    r.row_step = (long long)stride * 2;
    r.stage_step = (long long)rps * stride * 2;
    r.src = reinterpret_cast<const uint8_t*>(mat[m] + row * stride + col0);
    if (n < 1 || row < 0 || row + (long long)n * rps > mat_rows || col0 < 0 || col0 + S > stride ||
        (uint32_t)r.copies * r.bytes > (uint32_t)STAGE_BYTES ||
        ((reinterpret_cast<uintptr_t>(r.src) | r.bytes | (uint32_t)r.row_step) & 15u))
      return 0;  // the general path checks (and reports) each stage
    return n;
  }

  // Advance over a run of n stages returned by contiguous_run.
  __device__ __forceinline__ void skip_run(const KParams& p, int n) {
    if (chunks != 1) {  // whole rows in chunks, one matrix, within one expert's blocks
      const long long at = ((long long)j * groups + rg) * chunks + c + n;
      k += n;
      j = (int)(at / (groups * chunks));
      const int rem = (int)(at % (groups * chunks));
      rg = rem / chunks;
      c = rem % chunks;
      if (j == nblocks) {
        j = 0;
        ++es;
      }
      if (k < ns) row_base = block_row(p, j);
      return;
    }
    k += n;
    if (nmat == 1) {
      rg += n;
      j += rg / groups;
      rg %= groups;
      if (j == nblocks) {  // Mixtral expert ops: next selected expert
        j = 0;
        ++es;
      }
    } else {
      rg = 0;
      if (++m == nmat) {
        m = 0;
        if (++j == nblocks) {
          j = 0;
          ++es;
        }
      }
    }
    if (k < ns) row_base = block_row(p, j);
  }

  // Move to the next stage without issuing anything.
  __device__ __forceinline__ void advance(const KParams& p) {
    if (op != OP_PARTIAL && ++c == chunks) {
      c = 0;
      if (++rg == groups) {
        rg = 0;
        if (++m == nmat) {
          m = 0;
          if (++j == nblocks) {  // Mixtral expert ops: next selected expert
            j = 0;
            ++es;
          }
          if (k + 1 < ns) row_base = block_row(p, j);
        }
      }
    }
    ++k;
  }
};

// ------------------------------------------------------------------ ring
struct Ring {
  uint8_t* stages;
  uint64_t* full;
  uint64_t* empty;
  int slot;         // loader: next slot to fill
  uint32_t phase;   // loader: its phase parity
  uint32_t g;       // consumers: index of the next stage in this queue's stream
};


// Bounded wait on an mbarrier phase; false after ~timeout (then the engine is
// broken and the caller leaves the kernel).
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && (long long)(globaltimer() - t0) > timeout_ns) return false;
  }
}

__device__ __forceinline__ void ring_advance(Ring& r) {
  if (++r.slot == NUM_STAGES) {
    r.slot = 0;
    r.phase ^= 1u;
  }
}

}  // namespace ek
