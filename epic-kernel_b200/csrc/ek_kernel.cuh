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

namespace ek {

constexpr int CW = 8;                 // consumer warps
constexpr int NC = CW * 32;           // consumer threads
constexpr int NTHREADS = NC + 32;     // + loader warp
constexpr int STAGE_BYTES = 16384;    // one ring stage
constexpr int HALF_STAGE = 8192;      // one TMA box (16 rows x 256 bf16, or TK x D bf16)
constexpr int ACT_BYTES = 49152;      // activation vector + per-stage partial sums / attention merge
constexpr int NUM_STAGES = 11;        // 176 KiB ring
constexpr int CTRL_BYTES = 1024;      // mbarriers + reduction scratch
constexpr int SMEM_BYTES = NUM_STAGES * STAGE_BYTES + ACT_BYTES + CTRL_BYTES;
constexpr int GEMV_STAGE_COLS = 512;  // weight columns per stage (two 256-col boxes)
constexpr int MAX_GQA = 4;  // query heads per KV head

enum Op : int {
  OP_NOOP = 0,
  OP_QKV = 1,
  OP_PARTIAL = 2,
  OP_REDUCTION = 3,
  OP_OPROJ = 4,
  OP_UPGATE = 5,
  OP_DOWN = 6,
  OP_LM_HEAD = 7,
};

// Device status record; layout of EkStatus followed by the abort word.
struct DevStatus {
  int code, sm, instr, opcode, layer, observed, expected, detail;
  unsigned abort_epoch;  // == current epoch once any block failed in this launch
  int pad[7];
};

struct KParams {
  CUtensorMap tm_qkv, tm_o, tm_up, tm_gate, tm_down, tm_lm, tm_k, tm_v;

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

  int L, H, I, D, Hq, Hkv, V, T, rope_rows, maxP, brow, bcol, nq, Q;
  int qkv_rows, gqa, tk;
  int pos, skip_red;
  float scale, eps;
  int down_R, o_R, down_splits, o_splits;
  int pf_stages, record;
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

__device__ __forceinline__ int stages_per_row_block(int K) {
  return (K + GEMV_STAGE_COLS - 1) / GEMV_STAGE_COLS;
}

// Bytes of `act` a GEMV instruction needs: its activation slice (K bf16) and
// one 16-float partial row per ring stage.
__device__ __forceinline__ int gemv_act_bytes(int K, int ns) {
  return ((K * 2 + 15) & ~15) + ns * 64;
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
template <bool PREFETCH>
__device__ __forceinline__ uint32_t do_stage(const KParams& p, const Ins& ins, const Plan& pl, int k,
                                             uint8_t* dst, uint64_t* bar) {
  const int* w = ins.w;
  const CUtensorMap* map = nullptr;
  int K = 0, row = 0, col = 0;
  switch (pl.op) {
    case OP_QKV: {
      const int spb = stages_per_row_block(p.H);
      map = &p.tm_qkv;
      K = p.H;
      row = w[1] * p.qkv_rows + (w[2] + k / spb) * 16;
      col = (k % spb) * GEMV_STAGE_COLS;
      break;
    }
    case OP_OPROJ:
    case OP_DOWN: {
      const bool o = pl.op == OP_OPROJ;
      const int R = o ? p.o_R : p.down_R;
      const int spb = stages_per_row_block(R);
      map = o ? &p.tm_o : &p.tm_down;
      K = (w[4] + 1) * R;
      row = w[1] * p.H + (w[2] + k / spb) * 16;
      col = w[4] * R + (k % spb) * GEMV_STAGE_COLS;
      break;
    }
    case OP_UPGATE: {
      const int spb = stages_per_row_block(p.H);
      const int j = k / (2 * spb);
      const int r = k % (2 * spb);
      map = r < spb ? &p.tm_up : &p.tm_gate;
      K = p.H;
      row = w[1] * p.I + w[3 + j] * 16;
      col = (r % spb) * GEMV_STAGE_COLS;
      break;
    }
    case OP_LM_HEAD: {
      const int spb = stages_per_row_block(p.H);
      map = &p.tm_lm;
      K = p.H;
      row = (w[1] + k / spb) * 16;
      col = (k % spb) * GEMV_STAGE_COLS;
      break;
    }
    case OP_PARTIAL: {
      TokenRange r = partial_tokens(p, w[3], w[4]);
      const int t0 = w[1] * p.T + r.t_begin + k * p.tk;
      if (PREFETCH) {
        tma_prefetch_3d(&p.tm_k, 0, w[2], t0);
        tma_prefetch_3d(&p.tm_v, 0, w[2], t0);
      } else {
        mbar_arrive_expect_tx(bar, 2 * HALF_STAGE);
        tma_load_3d(dst, &p.tm_k, 0, w[2], t0, bar);
        tma_load_3d(dst + HALF_STAGE, &p.tm_v, 0, w[2], t0, bar);
      }
      return 2 * HALF_STAGE;
    }
    default:
      return 0;
  }
  const bool two = col + 256 < K;
  if (PREFETCH) {
    tma_prefetch_2d(map, col, row);
    if (two) tma_prefetch_2d(map, col + 256, row);
  } else {
    mbar_arrive_expect_tx(bar, two ? 2 * HALF_STAGE : HALF_STAGE);
    tma_load_2d(dst, map, col, row, bar);
    if (two) tma_load_2d(dst + HALF_STAGE, map, col + 256, row, bar);
  }
  return two ? 2 * HALF_STAGE : HALF_STAGE;
}

// ------------------------------------------------------------------ errors
__device__ __forceinline__ bool aborted(const KParams& p) {
  return ld_relaxed(reinterpret_cast<const int*>(&p.status->abort_epoch)) == (int)p.epoch;
}

__device__ inline void record_error(const KParams& p, int code, int instr, int opcode, int layer,
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
