// Batch-1 decode megakernel: loader and consumer roles, the opcode bodies,
// and the host-side launcher of one kernel variant. This file is compiled
// once per variant (EK_MODEL, EK_PF, and the namespace EK_NS of the kernel and
// its launcher are set on the command line; see ek_kernel.cuh).
//
// Opcode semantics follow megakernels/demos/latency/python_vm.py of
// epic-kernel (cited per op); see ek_kernel.cuh for the overall design.
#include <cuda_runtime.h>

#include <atomic>

#include "ek_kernel.cuh"
#include "ek_launch.h"

#ifndef EK_NS
#define EK_NS llama
#endif

namespace ek {
namespace {  // device code of this variant (internal linkage: one copy per variant)

// ------------------------------------------------------------------ GEMV streaming
// The GEMV inner loop, as free functions taking the ring state by value (so the
// consumer's state stays in registers; one out-of-line copy per variant).
//
// A stage holds RPS row segments of `len` columns (row i at st + i * len * 2);
// consumer thread t takes its 16-byte pieces t + 256 j (j < 4), whose column
// piece within the row is pc[j] and whose row is rowj[j] (warp-uniform:
// len % 256 == 0). Each thread keeps one fp32 accumulator per row of the 16-row
// block; at the end of the block the warp reduce-scatters the 16 rows and
// writes part[blk * BLOCK_PART + row * CW + warp]. Fixed summation order:
// within a thread, stages and pieces in stream order; then a fixed shuffle
// tree; then warps in order (row_sum).

// Bounded wait for a ring stage, per thread (no warp vote on the fast path):
// the clock is read only every 1024 polls. On timeout the thread records the
// stall, marks itself broken and stops waiting on the ring.
__device__ __forceinline__ void stage_wait(const KParams& p, uint64_t* bar, uint32_t parity, long long timeout,
                                           uint32_t& broken, int iidx, int slot) {
  if (broken || mbar_try_wait(bar, parity)) return;
  uint64_t t0 = 0;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return;
    if ((it & 1023u) == 0) {
      const uint64_t now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if ((long long)(now - t0) > timeout) {
        record_error(p, 4, iidx, -1, -1, slot, (int)parity, threadIdx.x >> 5);
        broken = 1;
        return;
      }
    }
  }
}

// RPS: rows per stage. ROW_IS_J: S == 2048, so piece j of every thread lies in
// row j of the stage at column piece tid. FULL: every stage holds 1024 pieces.
// Only RPS == 1 splits rows into column chunks.
#ifdef EK_GEMV_INLINE
#define EK_GEMV_LINKAGE __forceinline__
#else
#define EK_GEMV_LINKAGE __noinline__
#endif
template <int RPS, bool ROW_IS_J, bool FULL>
__device__ EK_GEMV_LINKAGE uint2 gemv_blocks_rps(const KParams& p, const uint8_t* stages, uint64_t* full,
                                              uint64_t* empty, uint32_t g, uint32_t broken, const uint8_t* act,
                                              int nblk, int chunks, int S, int x_base, float* part,
                                              uint32_t timing, int iidx) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ppr = min(S, STAGE_BYTES / 2) / 8;
  int pc[4], rowj[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int P = tid + 256 * j;
    rowj[j] = (RPS == 1 || ROW_IS_J) ? 0 : P / ppr;
    pc[j] = RPS == 1 ? P : ROW_IS_J ? tid : P - rowj[j] * ppr;
  }
  const long long ring_timeout = 4 * p.timeout_ns + 2000000000ll;
  uint32_t slot = g % NUM_STAGES, parity = (g / NUM_STAGES) & 1u;
  const uint4* xs4 = reinterpret_cast<const uint4*>(act) + x_base / 8;
  const int nch = RPS == 1 ? chunks : 1;
  int k = 0;
  for (int blk = 0; blk < nblk; ++blk) {
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll
    for (int rg = 0; rg < 16 / RPS; ++rg) {
      for (int c = 0; c < nch; ++c, ++k) {
        stage_wait(p, &full[slot], parity, ring_timeout, broken, iidx, (int)slot);
        if (timing != 0xffffffffu && tid == 0 && k < 28) {
          const int now = (int)(globaltimer() & 0x7fffffff);
          p.timings[(size_t)timing * 128 + TS_STAGE_USE + k] = now;
          if (k == 0) p.timings[(size_t)timing * 128 + TS_FIRST_USE] = now;
        }
        const uint4* w4 = reinterpret_cast<const uint4*>(stages + (size_t)slot * STAGE_BYTES);
        const int x0 = c * (STAGE_BYTES / 2);
        const int npieces = FULL ? 1024 : RPS * (min(STAGE_BYTES / 2, S - x0) / 8);
        const uint4* xc = xs4 + x0 / 8;
        // explicit shared-memory loads (the pointers arrive as generic
        // addresses); the activation piece is shared by the 4 rows of a stage
        // when ROW_IS_J
        const uint32_t wbase = smem_u32(w4), xbase = smem_u32(xc);
        uint4 xrow = make_uint4(0, 0, 0, 0);
        if (ROW_IS_J) xrow = lds128(xbase + pc[0] * 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (!FULL && tid + 256 * j >= npieces) continue;  // warp-uniform
          const uint4 wv = lds128(wbase + (tid + 256 * j) * 16);
          const uint4 xv = ROW_IS_J ? xrow : lds128(xbase + pc[j] * 16);
          const float d = dot8_bf16(wv, xv, 0.f);
          if (RPS == 1) {
            acc[rg] += d;
          } else if (ROW_IS_J) {
            acc[rg * RPS + j] += d;
          } else {
#pragma unroll
            for (int q = 0; q < RPS; ++q) acc[rg * RPS + q] += rowj[j] == q ? d : 0.f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == NUM_STAGES) {
          slot = 0;
          parity ^= 1u;
        }
      }
    }
    // reduce-scatter: after 4 halving levels lane l holds row l >> 1
#pragma unroll
    for (int lvl = 0; lvl < 4; ++lvl) {
      const int half = 8 >> lvl;
      const int off = 16 >> lvl;
      const bool up = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i >= half) break;
        const float send = up ? acc[i] : acc[i + half];
        const float keep = up ? acc[i + half] : acc[i];
        acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
    const float v = acc[0] + __shfl_xor_sync(0xffffffffu, acc[0], 1);
    if ((lane & 1) == 0) part[blk * BLOCK_PART + (lane >> 1) * CW + warp] = v;
  }
  return make_uint2(g + (uint32_t)k, broken);
}

// Returns (ring index after the instruction's stages, broken flag).
__device__ __forceinline__ uint2 gemv_blocks(const KParams& p, const uint8_t* stages, uint64_t* full,
                                             uint64_t* empty, uint32_t g, bool broken, const uint8_t* act,
                                             int nblk, int S, int x_base, float* part, uint32_t timing,
                                             int iidx) {
  const GemvShape sh = gemv_shape(S);
  const uint32_t b = broken ? 1u : 0u;
#define EK_GEMV(R, J, F) \
  gemv_blocks_rps<R, J, F>(p, stages, full, empty, g, b, act, nblk, sh.chunks, S, x_base, part, timing, iidx)
  switch (sh.rps) {
    case 16: return S == 512 ? EK_GEMV(16, false, true) : EK_GEMV(16, false, false);
    case 8: return S == 1024 ? EK_GEMV(8, false, true) : EK_GEMV(8, false, false);
    case 4: return S == 2048 ? EK_GEMV(4, true, true) : EK_GEMV(4, false, false);
    case 2: return S == 4096 ? EK_GEMV(2, false, true) : EK_GEMV(2, false, false);
    default: return S % 8192 == 0 ? EK_GEMV(1, false, true) : EK_GEMV(1, false, false);
  }
#undef EK_GEMV
}

// ------------------------------------------------------------------ consumer helpers
struct Consumer {
  const KParams& p;
  Ring ring;
  uint8_t* act;     // ACT_BYTES: bf16 activation vector or attention merge area
  float* red;       // CW floats of reduction scratch
  int* flag;        // one int broadcast between consumer threads
  // Mixtral: experts handed to the loader (mbox, completion on mbox_bar) and
  // router scratch (logits / probabilities, selected experts and scores)
  int* mbox;
  uint64_t* mbox_bar;
  float* rlog;
  int* rsel;
  float* rscore;
  int tid, warp, lane;
  int qidx, iidx;   // queue and instruction index (error reports, timings)
  // The ring stalled (an engine bug, reported as EK_STATUS_RING_TIMEOUT). A
  // broken warp stops waiting on the ring but keeps the same control flow, so
  // every named barrier is still reached by all consumer warps.
  bool broken;

  __device__ Consumer(const KParams& p_) : p(p_) {}

  __device__ __forceinline__ void sync() { named_sync<NC>(); }

  // Ring stages are numbered in stream order (ring.g); stage g lives in slot
  // g % NUM_STAGES with phase parity (g / NUM_STAGES) & 1. Every consumer warp
  // reads every stage and arrives once on its empty barrier (count CW).
  __device__ __forceinline__ const uint8_t* wait_stage(uint32_t g) {
    const int slot = g % NUM_STAGES;
    if (!broken) {
      const bool ok = ring_wait(&ring.full[slot], (g / NUM_STAGES) & 1u, 4 * p.timeout_ns + 2000000000ll);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) record_error(p, 4, iidx, -1, -1, slot, (int)((g / NUM_STAGES) & 1u), warp);
        broken = true;
      }
    }
    return ring.stages + (size_t)slot * STAGE_BYTES;
  }

  // Shared stage: every consumer warp calls acquire/release for it.
  __device__ __forceinline__ const uint8_t* acquire() { return wait_stage(ring.g); }

  __device__ __forceinline__ void release() {
    __syncwarp();
    if (lane == 0) mbar_arrive(&ring.empty[ring.g % NUM_STAGES]);
    ++ring.g;
  }

  // Skip ns stages without computing (aborted launch).
  __device__ void drain(int ns) {
    for (int k = 0; k < ns; ++k) {
      acquire();
      release();
    }
  }

  // Publication rule: every consumer thread writes its results, the consumer
  // warps pass a named barrier, then thread 0 bumps the counter with
  // red.release.gpu. Release is cumulative over the barrier, so readers that
  // acquire the counter see all those writes (they read with ld.global.cg).
  //
  // Thread 0 spins until every counter in `addrs` reaches its target, bounded
  // by p.timeout_ns. Returns (to all consumer threads) whether to run the op.
  __device__ bool wait_counters(int n, int* const* addrs, const int* targets, int opcode, int layer,
                                bool sys_scope = false) {
    if (n > 0) stamp(TS_WAIT);
    if (tid == 0) {
      int ok = 1;
      for (int j = 0; j < n && ok; ++j) {
        int v = sys_scope ? ld_acquire_sys(addrs[j]) : ld_acquire(addrs[j]);
        if (v >= targets[j]) continue;
        const uint64_t t0 = globaltimer();
        for (uint32_t it = 0;; ++it) {
          v = sys_scope ? ld_acquire_sys(addrs[j]) : ld_acquire(addrs[j]);
          if (v >= targets[j]) break;
          if ((it & 15u) == 15u) {
            if (aborted(p)) { ok = 0; break; }
            if ((long long)(globaltimer() - t0) > p.timeout_ns) {
              // detail: index into `barriers`, or -1 for a tensor-parallel
              // counter in a symmetric buffer
              record_error(p, 1, iidx, opcode, layer, v, targets[j],
                           sys_scope ? -1 : (int)(addrs[j] - p.barriers));
              ok = 0;
              break;
            }
          }
          __nanosleep(32);
        }
      }
      if (ok && aborted(p)) ok = 0;
      *flag = ok;
    }
    sync();
    const bool ok = *flag != 0;
    sync();
    return ok;
  }

  __device__ __forceinline__ int* bar(int layer, int row, int col) const {
    return p.barriers + ((size_t)layer * p.brow + row) * p.bcol + col;
  }

  __device__ __forceinline__ void stamp(int slot) {
    if (p.record && tid == 0 && p.timings) {
      int* t = p.timings + ((size_t)qidx * p.Q + iidx) * 128;
      const int now = (int)(globaltimer() & 0x7fffffff);
      t[slot] = now;
      if (slot == TS_STORE) t[TS_LAST_USE] = now;  // the GEMV stages end where the epilogue begins
    }
  }

  // Norm weights a thread needs (its pieces c = tid, tid + NC), loaded before
  // the counter wait so that their latency overlaps it.
  struct NormWeights {
    uint4 w[2];
  };
  __device__ __forceinline__ NormWeights preload_norm(const __nv_bfloat16* wt, int n) const {
    NormWeights r;
    const uint4* w4 = reinterpret_cast<const uint4*>(wt);
#pragma unroll
    for (int k = 0; k < 2; ++k) r.w[k] = tid + k * NC < n / 8 ? __ldg(w4 + tid + k * NC) : make_uint4(0, 0, 0, 0);
    return r;
  }

  // The residual stream entering layer 0: hidden_states, or the embedding
  // row of the input token (fused gather; a token outside the vocabulary is
  // reported and row 0 used, so the launch drains without faulting).
  __device__ __forceinline__ const __nv_bfloat16* layer0_input() const {
    if (!p.in_token) return p.hidden;
    long long t = __ldcg(p.in_token);
    if (t < 0 || t >= p.V) {
      if (tid == 0) record_error(p, 3, iidx, OP_QKV, 0, (int)t, p.V, -3);
      t = 0;
    }
    return p.embed + (size_t)t * p.H;
  }

  // Deferred down partials of layer `prev_layer` to add to the residual
  // stream (defer_down), or 0.
  __device__ __forceinline__ int deferred_splits(int prev_layer) const {
    return (prev_layer >= 0 && prev_layer < p.defer_down) ? p.down_splits : 0;
  }
  __device__ __forceinline__ const __nv_bfloat16* down_partials() const {
    return p.split_partials + (size_t)p.o_splits * p.H;
  }

  // 8 residual values at piece c of `x`, plus the nsplit deferred down
  // partials added in split order (bf16 rounding after each add).
  __device__ __forceinline__ uint4 residual8(const __nv_bfloat16* x, int c, int nsplit) const {
    uint4 v = __ldcg(reinterpret_cast<const uint4*>(x) + c);
    if (nsplit == 0) return v;
    uint4 parts[8];
    const uint4* d4 = reinterpret_cast<const uint4*>(down_partials());
#pragma unroll
    for (int j = 0; j < 8; ++j) if (j < nsplit) parts[j] = __ldcg(d4 + (size_t)j * (p.H / 8) + c);
    float h[8];
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) { h[2 * k] = bf_lo(u[k]); h[2 * k + 1] = bf_hi(u[k]); }
    auto add = [&](const uint4& pv) {
      const uint32_t q[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        h[2 * k] = bf16r(h[2 * k] + bf_lo(q[k]));
        h[2 * k + 1] = bf16r(h[2 * k + 1] + bf_hi(q[k]));
      }
    };
#pragma unroll
    for (int j = 0; j < 8; ++j) if (j < nsplit) add(parts[j]);
    for (int j = 8; j < nsplit; ++j) add(__ldcg(d4 + (size_t)j * (p.H / 8) + c));
    return make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]),
                      pack_bf16x2(h[6], h[7]));
  }

  // Residual-stream value of one row: hidden plus the nsplit deferred down
  // partials, in split order.
  __device__ __forceinline__ float residual_value(const __nv_bfloat16* x, int row, int nsplit) const {
    float h = ldcg_bf16(x + row);
    if (nsplit == 0) return h;
    const __nv_bfloat16* d = down_partials() + row;
    float parts[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) if (j < nsplit) parts[j] = ldcg_bf16(d + (size_t)j * p.H);
#pragma unroll
    for (int j = 0; j < 8; ++j) if (j < nsplit) h = bf16r(h + parts[j]);
    for (int j = 8; j < nsplit; ++j) h = bf16r(h + ldcg_bf16(d + (size_t)j * p.H));
    return h;
  }

  // xs[i] = bf16(w[i] * bf16(x[i] * rsqrt(mean(x^2) + eps))) for the n-vector at
  // `x` (python_vm.py:50-56), x being the residual stream with `nsplit`
  // deferred down partials added. Leaves xs in `act`.
  __device__ void rmsnorm_to_act(const __nv_bfloat16* x, const __nv_bfloat16* wt, int n, NormWeights nw,
                                 int nsplit = 0) {
    uint4* xs4 = reinterpret_cast<uint4*>(act);
    const uint4* w4 = reinterpret_cast<const uint4*>(wt);
    float ss = 0.f;
#pragma unroll 1
    for (int c = tid; c < n / 8; c += NC) {
      uint4 v = residual8(x, c, nsplit);
      xs4[c] = v;
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = bf_lo(u[k]), b = bf_hi(u[k]);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    sync();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < CW; ++k) tot += red[k];
    const float r = 1.0f / sqrtf(tot / (float)n + p.eps);
#pragma unroll 1
    for (int c = tid, k = 0; c < n / 8; c += NC, ++k) {
      const uint4 v = xs4[c];
      const uint4 g = k == 0 ? nw.w[0] : k == 1 ? nw.w[1] : __ldg(w4 + c);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float lo = bf_lo(gw[k]) * bf16r(bf_lo(u[k]) * r);
        const float hi = bf_hi(gw[k]) * bf16r(bf_hi(u[k]) * r);
        o[k] = pack_bf16x2(lo, hi);
      }
      xs4[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    sync();
  }

  // Copy n bf16 (n % 8 == 0) from global to act (values other SMs wrote).
  __device__ void copy_to_act(const __nv_bfloat16* x, int n) {
    uint4* xs4 = reinterpret_cast<uint4*>(act);
    const uint4* x4 = reinterpret_cast<const uint4*>(x);
    for (int c = tid; c < n / 8; c += NC) xs4[c] = __ldcg(x4 + c);
    sync();
  }

  // Stream the ns GEMV stages of the current instruction (whole 16-row blocks
  // of S-column row segments; the activation segment staged at
  // act[x_base .. x_base + S)). Block b's partials go to part[b * BLOCK_PART ..].
  // Returns after a consumer barrier, so the epilogue may read every partial.
  __device__ __forceinline__ void gemv_stream(int ns, int S, float* part, int x_base = 0) {
    const GemvShape g = gemv_shape(S);
    const int nblk = ns / ((16 / g.rps) * g.chunks);
    const uint32_t timing = (p.record && p.timings) ? (uint32_t)(qidx * p.Q + iidx) : 0xffffffffu;
    const uint2 r = gemv_blocks(p, ring.stages, ring.full, ring.empty, ring.g, broken, act, nblk, S, x_base, part,
                                timing, iidx);
    ring.g = r.x;
    broken = r.y != 0;
    sync();
  }

  __device__ __forceinline__ float* partials_after(int K) const {
    return reinterpret_cast<float*>(act + ((K * 2 + 15) & ~15));
  }

  // Row r of the 16-row block whose stages start at stage `first` (warps in
  // order).
  __device__ __forceinline__ static float row_sum(const float* part, int first, int S, int r) {
    const float* ps = part + (size_t)(first / stages_per_row_block(S)) * BLOCK_PART + r * CW;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < CW; ++w) v += ps[w];
    return v;
  }

  // ---------------------------------------------------------------- opcodes
  // LayerNorm_QKV_MatVecRopeAppend (python_vm.py:182-262).
  __device__ void op_qkv(const Ins& ins, const Plan& pl) {
    const int l = ins.w[1], b0 = ins.w[2], b1 = ins.w[3];
    const int qdim = p.Hq * p.D, kdim = p.Hkv * p.D;
    // loads that do not depend on other SMs, issued before the wait
    const NormWeights nw = preload_norm(p.attn_ln + (size_t)l * p.H, p.H);
    float2 rc = make_float2(1.f, 0.f), rs = make_float2(0.f, 0.f);
    {
      const int idx = tid;  // first rotary pair of this thread (the epilogue's first iteration)
      const int row = (b0 + idx / 8) * 16 + 2 * (idx % 8);
      if (idx < (b1 - b0) * 8 && row < qdim + kdim) {
        const int seg = row % p.D;
        rc = *reinterpret_cast<const float2*>(p.rope_cos + (size_t)p.pos * p.D + seg);
        rs = *reinterpret_cast<const float2*>(p.rope_sin + (size_t)p.pos * p.D + seg);
      }
    }
    if (l > 0) {
      int* a = bar(l - 1, OP_DOWN - 1, 0);
      const int t = p.down_done_target;
      if (!wait_counters(1, &a, &t, OP_QKV, l)) { drain(pl.ns); return; }
    } else if (!wait_counters(0, nullptr, nullptr, OP_QKV, l)) {  // abort check, CTA-uniform
      drain(pl.ns);
      return;
    }
    stamp(TS_READY);
    rmsnorm_to_act(l == 0 ? layer0_input() : p.hidden, p.attn_ln + (size_t)l * p.H, p.H, nw,
                   deferred_splits(l - 1));
    stamp(TS_ACT);
    const int spb = stages_per_row_block(p.H);
    float* part = partials_after(p.H);
    gemv_stream(pl.ns, p.H, part);
    stamp(TS_STORE);
    // one thread per rotary pair (rows 2i, 2i + 1 of a block)
#pragma unroll 1
    for (int idx = tid; idx < (b1 - b0) * 8; idx += NC) {
      const int j = idx / 8, pr = idx % 8;
      const int row = (b0 + j) * 16 + 2 * pr;
      float v0 = bf16r(row_sum(part, j * spb, p.H, 2 * pr));
      float v1 = bf16r(row_sum(part, j * spb, p.H, 2 * pr + 1));
      if (row < qdim + kdim) {
        // interleaved RoPE (llama.py:136-174) in fp32, rounded to bf16 on store
        if (idx != tid) {
          const int seg = row % p.D;
          rc = *reinterpret_cast<const float2*>(p.rope_cos + (size_t)p.pos * p.D + seg);
          rs = *reinterpret_cast<const float2*>(p.rope_sin + (size_t)p.pos * p.D + seg);
        }
        const float o0 = __fadd_rn(__fmul_rn(v0, rc.x), __fmul_rn(-v1, rs.x));
        const float o1 = __fadd_rn(__fmul_rn(v1, rc.y), __fmul_rn(v0, rs.y));
        v0 = o0;
        v1 = o1;
      }
      __nv_bfloat16* dst;
      if (row < qdim) {
        dst = p.q + row;
      } else if (row < qdim + kdim) {
        dst = p.k_cache + ((size_t)l * p.T + p.pos) * kdim + (row - qdim);
      } else {
        dst = p.v_cache + ((size_t)l * p.T + p.pos) * kdim + (row - qdim - kdim);
      }
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(v0, v1);
    }
    sync();
    if (tid == 0) {
      const int bph = p.D / 16;
      int b = b0;
      while (b < b1) {
        const int head = b / bph;
        int cnt = 0;
        while (b < b1 && b / bph == head) { ++cnt; ++b; }
        red_release_add(bar(l, OP_QKV - 1, head), cnt);
      }
    }
  }

  // Attention over a ring stage of TK tokens (K rows at st, V rows at
  // st + HALF_STAGE, D bf16 each): warp w takes tokens [w * TPW, w * TPW + TPW).
  // Lanes have two roles per tile.
  // - score role: lane = (token * MAX_GQA + head) * LPP + half computes the
  //   q . k dot over D / LPP dims, q held in registers as bf16 (qr). Chunks are
  //   read in an order rotated by (token * LPP + half) so that the lanes of a
  //   warp hit distinct shared-memory banks; qr is stored in the same rotation.
  // - output role: lane = group * MAX_GQA + head accumulates VD = D / 8 output
  //   dims [group * VD, group * VD + VD) of its head; its token weights come
  //   from the score lanes by shuffles.
  // The warp keeps an online softmax per head over its own tokens (one max and
  // one sum reduction per tile); warps are merged at the end.
  template <int D>
  struct AttnRoles {
    static constexpr int TK = HALF_STAGE / (D * 2);   // tokens per stage
    static constexpr int TPW = TK / CW;               // tokens per warp per stage
    static constexpr int LPP = 32 / (TPW * MAX_GQA);  // lanes per (token, head)
    static constexpr int DPL = D / LPP;               // dims per score lane
    static constexpr int NQ = DPL / 8;                // 16-byte chunks per score lane
    static constexpr int VD = MAX_GQA * D / 32;       // output dims per lane
    static_assert(LPP >= 1 && LPP * TPW * MAX_GQA == 32, "lane roles");
  };

  template <int D>
  __device__ __forceinline__ void attend_tile(const uint8_t* kb, const uint8_t* vb, int nvalid, bool global,
                                              const uint4 (&qr)[AttnRoles<D>::NQ], float& ms, float& ls,
                                              float (&acc)[AttnRoles<D>::VD], int gqa) {
    using R = AttnRoles<D>;
    const int pair = lane / R::LPP, half = lane % R::LPP;
    const int stok = pair / MAX_GQA, sh = pair % MAX_GQA;
    const int oh = lane % MAX_GQA, od0 = (lane / MAX_GQA) * R::VD;
    const bool sv = stok < nvalid && sh < gqa;
    float d = 0.f;
    if (sv) {
      const int rot = stok * R::LPP + half;
      const uint4* k4 = reinterpret_cast<const uint4*>(kb + (size_t)stok * D * 2 + half * R::DPL * 2);
#pragma unroll
      for (int i = 0; i < R::NQ; ++i) {
        const int c = (i + rot) % R::NQ;
        const uint4 w = global ? __ldcg(k4 + c) : k4[c];
        d = dot8_bf16(w, qr[i], d);
      }
    }
#pragma unroll
    for (int o = 1; o < R::LPP; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    const float sc = sv ? d * p.scale : -INFINITY;
    float mt = sc;
#pragma unroll
    for (int o = MAX_GQA * R::LPP; o < 32; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
    const float mn = fmaxf(ms, mt);
    const float mref = mn == -INFINITY ? 0.f : mn;
    const float corr = expf(ms - mref);
    const float pe = sv ? expf(sc - mref) : 0.f;
    float ps = pe;
#pragma unroll
    for (int o = MAX_GQA * R::LPP; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    ls = ls * corr + ps;
    ms = mn;
    // output role: rescale, then add the tile's weighted V rows
    const float co = __shfl_sync(0xffffffffu, corr, oh * R::LPP);
#pragma unroll
    for (int e = 0; e < R::VD; ++e) acc[e] *= co;
    for (int t = 0; t < nvalid; ++t) {  // warp-uniform bound
      const float pt = __shfl_sync(0xffffffffu, pe, (t * MAX_GQA + oh) * R::LPP);
      const uint4* v4 = reinterpret_cast<const uint4*>(vb + (size_t)t * D * 2 + od0 * 2);
#pragma unroll
      for (int c = 0; c < R::VD / 8; ++c) {
        const uint4 v = global ? __ldcg(v4 + c) : v4[c];
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[c * 8 + 2 * q] = fmaf(pt, bf_lo(u[q]), acc[c * 8 + 2 * q]);
          acc[c * 8 + 2 * q + 1] = fmaf(pt, bf_hi(u[q]), acc[c * 8 + 2 * q + 1]);
        }
      }
    }
  }

  // PartialAttention (python_vm.py:291-357): softmax(q K^T * scale) V over the
  // partial's token slice for the query heads of one KV head; LSE is
  // log2(sum(exp(scores))).
  template <int D>
  __device__ void op_partial(const Ins& ins, const Plan& pl) {
    using R = AttnRoles<D>;
    const int l = ins.w[1], kvh = ins.w[2], P = ins.w[3], part = ins.w[4];
    const int gqa = p.gqa, hs = kvh * gqa, bph = D / 16;
    {
      int* a[MAX_GQA + 2];
      int t[MAX_GQA + 2];
      for (int h = 0; h < gqa; ++h) { a[h] = bar(l, OP_QKV - 1, hs + h); t[h] = bph; }
      a[gqa] = bar(l, OP_QKV - 1, p.Hq + kvh);
      a[gqa + 1] = bar(l, OP_QKV - 1, p.Hq + p.Hkv + kvh);
      t[gqa] = t[gqa + 1] = bph;
      if (!wait_counters(gqa + 2, a, t, OP_PARTIAL, l)) { drain(pl.ns); return; }
    }
    stamp(TS_READY);
    const TokenRange tr = partial_tokens(p, P, part);
    // this lane's q chunks (score role), rotated like the K reads
    uint4 qr[R::NQ];
    {
      const int pair = lane / R::LPP, half = lane % R::LPP;
      const int stok = pair / MAX_GQA, sh = pair % MAX_GQA;
      const int rot = stok * R::LPP + half;
      const uint4* q4 = reinterpret_cast<const uint4*>(p.q + (size_t)(hs + (sh < gqa ? sh : 0)) * D + half * R::DPL);
#pragma unroll
      for (int i = 0; i < R::NQ; ++i) qr[i] = __ldcg(q4 + (i + rot) % R::NQ);
    }
    stamp(TS_ACT);
    float ms = -INFINITY, ls = 0.f, acc[R::VD];
#pragma unroll
    for (int e = 0; e < R::VD; ++e) acc[e] = 0.f;
    for (int k = 0; k < pl.ns; ++k) {
      const uint8_t* st = acquire();
      const int t0 = tr.t_begin + k * R::TK + warp * R::TPW;
      const int nvalid = max(0, min(R::TPW, tr.t_load_end - t0));
      if (nvalid > 0)
        attend_tile<D>(st + (size_t)warp * R::TPW * D * 2, st + HALF_STAGE + (size_t)warp * R::TPW * D * 2,
                       nvalid, false, qr, ms, ls, acc, gqa);
      release();
    }
    // the token appended by this step's QKV instructions is read from global
    if (warp == 0 && p.pos >= tr.t_begin && p.pos < tr.t_end) {
      const size_t off = (((size_t)l * p.T + p.pos) * p.Hkv + kvh) * D;
      attend_tile<D>(reinterpret_cast<const uint8_t*>(p.k_cache + off),
                     reinterpret_cast<const uint8_t*>(p.v_cache + off), 1, true, qr, ms, ls, acc, gqa);
    }
    stamp(TS_STORE);
    // merge the per-warp online-softmax states
    float* mm = reinterpret_cast<float*>(act);  // [CW][gqa]
    float* ll = mm + CW * MAX_GQA;              // [CW][gqa]
    float* aa = ll + CW * MAX_GQA;              // [CW][gqa][D]
    {
      const int oh = lane % MAX_GQA, od0 = (lane / MAX_GQA) * R::VD;
      // score lanes of token 0 hold each head's state
      if (lane < MAX_GQA * R::LPP && lane % R::LPP == 0 && lane / R::LPP < gqa) {
        mm[warp * gqa + lane / R::LPP] = ms;
        ll[warp * gqa + lane / R::LPP] = ls;
      }
      if (oh < gqa) {
#pragma unroll
        for (int e = 0; e < R::VD; ++e) aa[(warp * gqa + oh) * D + od0 + e] = acc[e];
      }
    }
    sync();
    for (int idx = tid; idx < gqa * D; idx += NC) {
      const int h = idx / D, d = idx % D;
      float M = -INFINITY;
      for (int w = 0; w < CW; ++w) M = fmaxf(M, mm[w * gqa + h]);
      float Ls = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int w = 0; w < CW; ++w) {
          const float f = expf(mm[w * gqa + h] - M);
          Ls = fmaf(ll[w * gqa + h], f, Ls);
          O = fmaf(aa[(w * gqa + h) * D + d], f, O);
        }
      }
      float out, lse;
      if (Ls > 0.f) {
        out = O / Ls;
        lse = log2f(Ls) + M * 1.4426950408889634f;
      } else {
        out = 0.f;
        lse = -INFINITY;
      }
      const int head = hs + h;
      if (p.skip_red) {
        p.attn_out[(size_t)head * D + d] = __float2bfloat16_rn(out);
      } else {
        p.attn_o[((size_t)head * p.maxP + part) * D + d] = out;
        if (d == 0) p.lse[(size_t)head * p.maxP + part] = lse;
      }
    }
    sync();
    if (p.skip_red) {
      if (tid == 0) red_release_add(bar(l, OP_REDUCTION - 1, 0), gqa);
      return;
    }
    if (!p.fuse_red) {
      if (tid == 0)
        for (int h = 0; h < gqa; ++h) red_release_add(bar(l, OP_PARTIAL - 1, hs + h), 1);
      return;
    }
    // fused reduction: the last partial of this KV head to arrive merges all P
    // partials (acquire-release on the head's counter orders the other
    // partials' writes before the merge's reads)
    if (tid == 0) {
      for (int h = 1; h < gqa; ++h) red_release_add(bar(l, OP_PARTIAL - 1, hs + h), 1);
      *flag = atom_add_acq_rel(bar(l, OP_PARTIAL - 1, hs), 1) == P - 1;
    }
    sync();
    const bool last = *flag != 0;
    sync();
    if (last) merge_partials(l, hs, P, nullptr, true, 0);
  }

  // AttentionReduction (python_vm.py:360-401): exp2-weighted merge of partials.
  __device__ void op_reduction(const Ins& ins) {
    if (p.fuse_red) return;  // merged by the last partial of each KV head
    const int l = ins.w[1], hs = ins.w[2], P = ins.w[3], terminal = ins.w[4], n = ins.w[5];
    {
      int* a = bar(l, OP_PARTIAL - 1, hs);
      if (!wait_counters(1, &a, &P, OP_REDUCTION, l)) return;
    }
    stamp(TS_READY);
    merge_partials(l, hs, n, ins.w + 6, terminal != 0, ins.w[6 + n]);
  }

  // Merge the n partials list[0..n) (identity when list is null) of the gqa
  // query heads starting at hs, and bump the layer's reduction counter. The
  // partials' LSEs are staged in shared memory first so that every load of
  // the merge is issued independently.
  __device__ void merge_partials(int l, int hs, int n, const int* list, bool terminal, int out_slot) {
    const int D = p.D, gqa = p.gqa;
    // [gqa][n] exp2(lse - max), n <= 160, past the partials' merge area
    float* fac = reinterpret_cast<float*>(act + ACT_BYTES - 4096);
    float* den = fac + MAX_GQA * 160;  // [gqa]
    for (int i = tid; i < gqa * n; i += NC) {
      const int h = i / n, j = i - h * n;
      fac[i] = __ldcg(p.lse + (size_t)(hs + h) * p.maxP + (list ? list[j] : j));
    }
    sync();
    if (tid < gqa) {
      float M = -INFINITY;
      for (int j = 0; j < n; ++j) M = fmaxf(M, fac[tid * n + j]);
      float s = 0.f;
      for (int j = 0; j < n; ++j) {
        const float f = exp2f(fac[tid * n + j] - M);
        fac[tid * n + j] = f;
        s += f;
      }
      den[tid] = s;
    }
    sync();
    // compute first, write after a barrier: the output slot may be an input
    float res[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = tid + k * NC;
      res[k] = 0.f;
      if (idx >= gqa * D) continue;
      const int h = idx / D, d = idx - h * D;
      const float* o = p.attn_o + (size_t)(hs + h) * p.maxP * D + d;
      float num = 0.f;
#pragma unroll 1
      for (int j0 = 0; j0 < n; j0 += 8) {
        float vals[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          vals[j] = j0 + j < n ? __ldcg(o + (size_t)(list ? list[j0 + j] : j0 + j) * D) : 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j0 + j < n) num = fmaf(vals[j], fac[h * n + j0 + j], num);
      }
      res[k] = num / den[h];
    }
    sync();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = tid + k * NC;
      if (idx >= gqa * D) continue;
      const int h = idx / D, d = idx - h * D;
      if (terminal) {
        p.attn_out[(size_t)(hs + h) * D + d] = __float2bfloat16_rn(res[k]);
      } else {
        const size_t row = (size_t)(hs + h) * p.maxP + out_slot;
        p.attn_o[row * D + d] = res[k];
        if (d == 0) p.lse[row] = logf(den[h]);
      }
    }
    sync();
    if (tid == 0) red_release_add(bar(l, OP_REDUCTION - 1, 0), gqa);
  }

  // Epoch-tagged arrival counter: returns the arrival number (1-based) of this
  // call in the current launch. Counters left by an aborted launch are stale
  // (different epoch) and restart at 1.
  __device__ __forceinline__ unsigned arrive_split(unsigned* ctr) {
    const unsigned tag = (p.epoch & 0xffffffu) << 8;
    unsigned old = *reinterpret_cast<volatile unsigned*>(ctr);
    while (true) {
      const unsigned nv = ((old & ~0xffu) == tag) ? old + 1 : (tag | 1u);
      const unsigned prev = atomicCAS(ctr, old, nv);
      if (prev == old) return nv & 0xffu;
      old = prev;
    }
  }

  // hidden[rows] += W[rows, split cols] . x  for O_ProjResidual / DownProjResidual
  // (python_vm.py:59-80, 101-139). With several column splits, each split
  // stores its bf16 partial; the last split to arrive for a 16-row block adds
  // the partials to hidden in split order, as the interpreter does.
  __device__ void op_matvec_add(const Ins& ins, const Plan& pl) {
    const bool o = pl.op == OP_OPROJ;
    const int l = ins.w[1], b0 = ins.w[2], b1 = ins.w[3], split = ins.w[4];
    const int R = o ? p.o_R : p.down_R;
    const int splits = o ? p.o_splits : p.down_splits;
    const int nrows = (b1 - b0) * 16;
    // O-proj adds into the residual stream: once layer l - 1 is complete (in
    // practice long before this layer's attention is), the first row of each
    // thread, with layer l - 1's deferred down partials, is read before the
    // attention wait, so that its latency overlaps the wait
    const bool own_rows = o && splits == 1 && p.tp_world <= 1;
    const int nsplit = own_rows ? deferred_splits(l - 1) : 0;
    const __nv_bfloat16* xres = l == 0 ? layer0_input() : p.hidden;
    float hpre = 0.f;
    if (own_rows) {
      if (l > 0) {  // the rows must hold layer l - 1's result (or its deferred partials)
        int* a = bar(l - 1, OP_DOWN - 1, 0);
        const int t = p.down_done_target;
        if (!wait_counters(1, &a, &t, pl.op, l)) { drain(pl.ns); return; }
      }
      if (tid < nrows) hpre = residual_value(xres, b0 * 16 + tid, nsplit);
    }
    {
      int* a = o ? bar(l, OP_REDUCTION - 1, 0) : bar(l, OP_UPGATE - 1, 0);
      const int t = o ? p.Hq : p.I / 16;
      if (!wait_counters(1, &a, &t, pl.op, l)) { drain(pl.ns); return; }
    }
    stamp(TS_READY);
    copy_to_act((o ? p.attn_out : p.silu) + (size_t)split * R, R);
    stamp(TS_ACT);
    // partial sums: [o_splits][H] for O_ProjResidual, then [down_splits][H]
    __nv_bfloat16* partials = p.split_partials + (size_t)(o ? 0 : p.o_splits) * p.H;
    const int spb = stages_per_row_block(R);
    float* part = partials_after(R);
    gemv_stream(pl.ns, R, part);
    stamp(TS_STORE);
    if (kMixtral && o && p.tp_world > 1) {
      // tensor parallel: all-reduce the fp32 row partials over NVLink, then
      // add their rank-ordered sum, rounded once, to hidden (same on all ranks)
      for (int idx = tid; idx < (b1 - b0) * 16; idx += NC) {
        const int j = idx / 16, r = idx % 16;
        const int row = (b0 + j) * 16 + r;
        const float v = row_sum(part, j * spb, R, r);
        for (int rk = 0; rk < p.tp_world; ++rk) tp_slot(rk, p.tp_off_recv_o)[(size_t)p.tp_rank * p.H + row] = v;
      }
      sync();
      if (!tp_exchange(p.tp_off_cnt_o, l, b0, b1, OP_OPROJ)) return;
      const float* recv = tp_slot(p.tp_rank, p.tp_off_recv_o);
      for (int idx = tid; idx < (b1 - b0) * 16; idx += NC) {
        const int row = b0 * 16 + idx;
        float sum = 0.f;
        for (int rk = 0; rk < p.tp_world; ++rk) sum += __ldcg(recv + (size_t)rk * p.H + row);
        p.hidden[row] = __float2bfloat16_rn(ldcg_bf16(p.hidden + row) + bf16r(sum));
      }
      sync();
      if (tid == 0) red_release_add(bar(l, OP_OPROJ - 1, 0), b1 - b0);
      return;
    }
#pragma unroll 1
    for (int idx = tid; idx < nrows; idx += NC) {
      const int j = idx / 16, r = idx % 16;
      const int row = (b0 + j) * 16 + r;
      const float v = bf16r(row_sum(part, j * spb, R, r));
      if (splits == 1) {
        const float h = own_rows && idx == tid ? hpre : residual_value(xres, row, nsplit);
        p.hidden[row] = __float2bfloat16_rn(h + v);
      } else {
        partials[(size_t)split * p.H + row] = __float2bfloat16_rn(v);
      }
    }
    sync();
    int* done = bar(l, pl.op - 1, 0);
    if (splits == 1 || (!o && l < p.defer_down)) {
      // one writer per row, or split partials left for the next layer's readers
      if (tid == 0) red_release_add(done, b1 - b0);
      return;
    }
    unsigned* ctrs = p.split_counters + ((size_t)l * 2 + (o ? 0 : 1)) * (p.H / 16);
    for (int b = b0 + warp; b < b1; b += CW) {
      unsigned arrival = 0;
      if (lane == 0) {
        __threadfence();
        arrival = arrive_split(ctrs + b);
      }
      arrival = __shfl_sync(0xffffffffu, arrival, 0);
      if (arrival == (unsigned)splits) {
        __threadfence();
        if (lane < 16) {
          const int row = b * 16 + lane;
          float h = ldcg_bf16(p.hidden + row);
          for (int c = 0; c < splits; ++c) h = bf16r(h + ldcg_bf16(partials + (size_t)c * p.H + row));
          p.hidden[row] = __float2bfloat16_rn(h);
        }
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          red_release_add(done, splits);
        }
      }
    }
  }

  // LayerNormDoubleMatVecSiLU (python_vm.py:142-179): silu(gate) * up per block.
  __device__ void op_upgate(const Ins& ins, const Plan& pl) {
    const int l = ins.w[1], n = ins.w[2];
    const NormWeights nw = preload_norm(p.mlp_ln + (size_t)l * p.H, p.H);
    {
      int* a = bar(l, OP_OPROJ - 1, 0);
      const int t = p.H / 16;
      if (!wait_counters(1, &a, &t, OP_UPGATE, l)) { drain(pl.ns); return; }
    }
    stamp(TS_READY);
    rmsnorm_to_act(p.hidden, p.mlp_ln + (size_t)l * p.H, p.H, nw);
    stamp(TS_ACT);
    const int spb = stages_per_row_block(p.H);
    float* part = partials_after(p.H);
    gemv_stream(pl.ns, p.H, part);
    stamp(TS_STORE);
    for (int idx = tid; idx < n * 16; idx += NC) {
      const int j = idx / 16, r = idx % 16;
      const float u = bf16r(row_sum(part, j * 2 * spb, p.H, r));
      const float gt = bf16r(row_sum(part, j * 2 * spb + spb, p.H, r));
      const float sl = bf16r(gt / (1.0f + expf(-gt)));
      p.silu[ins.w[3 + j] * 16 + r] = __float2bfloat16_rn(sl * u);
    }
    sync();
    if (tid == 0) red_release_add(bar(l, OP_UPGATE - 1, 0), n);
  }

  // RMS_LM_Head (python_vm.py:265-288): logits rows of the final RMSNorm'd hidden.
  __device__ void op_lm_head(const Ins& ins, const Plan& pl) {
    const int b0 = ins.w[1], b1 = ins.w[2];
    const NormWeights nw = preload_norm(p.lm_norm, p.H);
    {
      int* a = bar(p.L - 1, OP_DOWN - 1, 0);
      const int t = p.down_done_target;
      if (!wait_counters(1, &a, &t, OP_LM_HEAD, p.L - 1)) { drain(pl.ns); return; }
    }
    stamp(TS_READY);
    rmsnorm_to_act(p.hidden, p.lm_norm, p.H, nw);
    stamp(TS_ACT);
    const int spb = stages_per_row_block(p.H);
    float* part = partials_after(p.H);
    gemv_stream(pl.ns, p.H, part);
    stamp(TS_STORE);
    unsigned long long best = 0;  // argmax key of this thread's rows
    for (int idx = tid; idx < (b1 - b0) * 16; idx += NC) {
      const int j = idx / 16, r = idx % 16;
      const __nv_bfloat16 v = __float2bfloat16_rn(row_sum(part, j * spb, p.H, r));
      p.logits[(b0 + j) * 16 + r] = v;
      best = max(best, argmax_key(v, (b0 + j) * 16 + r));
    }
    if (p.out_token) finish_argmax(best);
  }

  // Argmax key: launch tag, bf16 value mapped to an unsigned order, then the
  // row complemented, so that the largest key is the largest value's first row
  // (torch.argmax's tie rule).
  __device__ __forceinline__ unsigned long long argmax_key(__nv_bfloat16 v, int row) const {
    unsigned b = __bfloat16_as_ushort(v);
    b = (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
    return ((unsigned long long)(p.epoch & 0xffffu) << 48) | ((unsigned long long)b << 32) |
           (unsigned long long)(0xffffffffu - (unsigned)row);
  }

  // Merge this instruction's best key into the launch's, count the
  // instruction, and let the last LM-head instruction write the token.
  __device__ void finish_argmax(unsigned long long best) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    // CW keys in the activation area (the GEMV that read it has finished)
    unsigned long long* wbest = reinterpret_cast<unsigned long long*>(act);
    if (lane == 0) wbest[warp] = best;
    sync();
    if (tid == 0) {
      for (int w = 0; w < CW; ++w) best = max(best, wbest[w]);
      atomicMax(&p.status->argmax_key, best);
      __threadfence();
      // this launch's arrival slot (cleared by block 0 of the previous launch)
      const unsigned n = atomicAdd(&p.status->lm_arrivals[p.epoch & 3u], 1u) + 1u;
      if ((int)n == p.lm_count) {
        __threadfence();
        const unsigned long long k = atomicMax(&p.status->argmax_key, 0ull);
        *p.out_token = (long long)(0xffffffffu - (unsigned)(k & 0xffffffffull));
      }
    }
    sync();
  }
  // ---------------------------------------------------------------- tensor parallel
  __device__ __forceinline__ float* tp_slot(int rank, long long off) const {
    return reinterpret_cast<float*>(p.tp_peer[rank] + off);
  }
  __device__ __forceinline__ int* tp_counter(int rank, long long off, int idx) const {
    return reinterpret_cast<int*>(p.tp_peer[rank] + off) + idx;
  }

  // Signal every rank that this rank pushed blocks [b0, b1) of layer l (one
  // counter per 16-row block), then wait until all ranks pushed them here.
  // Call after a consumer barrier that follows the pushes.
  __device__ bool tp_exchange(long long cnt_off, int l, int b0, int b1, int opcode) {
    // one system-scope release per (rank, block), issued in parallel by the
    // lanes of warp 0 (serially they cost one NVLink round trip each)
    if (warp == 0) {
      const int nb = b1 - b0;
      for (int k = lane; k < p.tp_world * nb; k += 32)
        red_release_sys_add(tp_counter(k / nb, cnt_off, l * (p.H / 16) + b0 + k % nb), 1);
    }
    bool ok = true;
    const int target = p.tp_world * (int)p.tp_step;
    for (int b = b0; b < b1 && ok; ++b) {
      int* a = tp_counter(p.tp_rank, cnt_off, l * (p.H / 16) + b);
      ok = wait_counters(1, &a, &target, opcode, l, true);
    }
    return ok;
  }

  // ---------------------------------------------------------------- Mixtral
  // Hand the experts of the current expert instruction to the loader (one
  // handoff per RmsRouterUpgate / ExpertDownProjFused with ring stages).
  __device__ __forceinline__ void handoff(const int* experts) {
    if (tid == 0) {
      for (int i = 0; i < p.topk; ++i) mbox[i] = experts[i];
      mbar_arrive(mbox_bar);
    }
  }

  // Router over the RMSNorm'd hidden in act[0..H) (python_vm.py:541-550):
  // fp32 logits, softmax, top-k (ties: lower index), scores renormalised over
  // the top k. Leaves rsel / rscore for every consumer thread.
  __device__ void router(int l) {
    const uint4* xs = reinterpret_cast<const uint4*>(act);
    for (int e = warp; e < p.E; e += CW) {
      const uint4* wr = reinterpret_cast<const uint4*>(p.w_router + ((size_t)l * p.E + e) * p.H);
      float d = 0.f;
      for (int c = lane; c < p.H / 8; c += 32) {
        const uint4 wv = __ldg(wr + c), xv = xs[c];
        d = fmaf(bf_lo(wv.x), bf_lo(xv.x), d);
        d = fmaf(bf_hi(wv.x), bf_hi(xv.x), d);
        d = fmaf(bf_lo(wv.y), bf_lo(xv.y), d);
        d = fmaf(bf_hi(wv.y), bf_hi(xv.y), d);
        d = fmaf(bf_lo(wv.z), bf_lo(xv.z), d);
        d = fmaf(bf_hi(wv.z), bf_hi(xv.z), d);
        d = fmaf(bf_lo(wv.w), bf_lo(xv.w), d);
        d = fmaf(bf_hi(wv.w), bf_hi(xv.w), d);
      }
      d = warp_sum(d);
      if (lane == 0) rlog[e] = d;
    }
    sync();
    if (tid == 0) {
      float mx = -INFINITY;
      for (int e = 0; e < p.E; ++e) mx = fmaxf(mx, rlog[e]);
      float sum = 0.f;
      for (int e = 0; e < p.E; ++e) {
        rlog[e] = expf(rlog[e] - mx);
        sum += rlog[e];
      }
      for (int e = 0; e < p.E; ++e) rlog[e] /= sum;
      float tot = 0.f;
      for (int i = 0; i < p.topk; ++i) {
        int best = -1;
        for (int e = 0; e < p.E; ++e) {
          bool taken = false;
          for (int q = 0; q < i; ++q) taken |= rsel[q] == e;
          if (!taken && (best < 0 || rlog[e] > rlog[best])) best = e;
        }
        rsel[i] = best;
        rscore[i] = rlog[best];
        tot += rlog[best];
      }
      for (int i = 0; i < p.topk; ++i) rscore[i] /= tot;
    }
    sync();
  }

  // RmsRouterUpgate (mixtral/python_vm.py:525-574).
  __device__ void op_router_upgate(const Ins& ins, const Plan& pl) {
    const int l = ins.w[1], b0 = ins.w[2], nb = ins.w[3];
    const NormWeights nw = preload_norm(p.ffn_ln + (size_t)l * p.H, p.H);
    {
      int* a = bar(l, OP_OPROJ - 1, 0);
      const int t = p.H / 16;
      if (!wait_counters(1, &a, &t, OP_UPGATE, l)) {
        const int fallback[MAX_TOPK] = {0, 1 % p.E, 2 % p.E, 3 % p.E};
        if (pl.ns > 0) handoff(fallback);
        drain(pl.ns);
        return;
      }
    }
    stamp(TS_READY);
    rmsnorm_to_act(p.hidden, p.ffn_ln + (size_t)l * p.H, p.H, nw);
    router(l);
    if (pl.ns > 0) handoff(rsel);
    if (tid < p.topk) {
      p.sel_idx[tid] = rsel[tid];
      p.sel_scores[tid] = __float2bfloat16_rn(rscore[tid]);
    }
    {
      const uint4* xs = reinterpret_cast<const uint4*>(act);
      for (int c = tid; c < p.H / 8; c += NC) reinterpret_cast<uint4*>(p.router_normed)[c] = xs[c];
    }
    stamp(TS_ACT);
    const int spb = stages_per_row_block(p.H);
    float* part = partials_after(p.H);
    gemv_stream(pl.ns, p.H, part);
    stamp(TS_STORE);
    for (int idx = tid; idx < p.topk * nb * 16; idx += NC) {
      const int es = idx / (nb * 16), j = (idx / 16) % nb, r = idx % 16;
      const int first = (es * nb + j) * 2 * spb;
      const float gt = bf16r(row_sum(part, first, p.H, r));
      const float up = bf16r(row_sum(part, first + spb, p.H, r));
      const float sl = bf16r(gt / (1.0f + expf(-gt)));
      p.expert_silu[(size_t)rsel[es] * p.I + (b0 + j) * 16 + r] = __float2bfloat16_rn(sl * up);
    }
    sync();
    if (tid == 0) red_release_add(bar(l, OP_UPGATE - 1, 0), nb);
  }

  // ExpertDownProjFused (mixtral/python_vm.py:581-611): per selected expert in
  // top-k order, hidden += bf16(score * bf16(W_down[e][rows] . silu[e])).
  __device__ void op_expert_down(const Ins& ins, const Plan& pl) {
    const int l = ins.w[1], b0 = ins.w[2], b1 = ins.w[3], nb = b1 - b0;
    {
      int* a = bar(l, OP_UPGATE - 1, 0);
      const int t = p.I / 16;
      if (!wait_counters(1, &a, &t, OP_DOWN, l)) {
        const int fallback[MAX_TOPK] = {0, 1 % p.E, 2 % p.E, 3 % p.E};
        if (pl.ns > 0) handoff(fallback);
        drain(pl.ns);
        return;
      }
    }
    stamp(TS_READY);
    if (tid < p.topk) {
      int e = __ldcg(p.sel_idx + tid);
      rsel[tid] = (e < 0 || e >= p.E) ? 0 : e;
      rscore[tid] = ldcg_bf16(p.sel_scores + tid);
    }
    sync();
    if (pl.ns > 0) handoff(rsel);
    const int spb = stages_per_row_block(p.I);
    const int nse = nb * spb;
    float* part = partials_after(p.I);
    for (int es = 0; es < p.topk; ++es) {
      copy_to_act(p.expert_silu + (size_t)rsel[es] * p.I, p.I);
      gemv_stream(nse, p.I, part + es * nb * BLOCK_PART);
    }
    stamp(TS_STORE);
    if (p.tp_world > 1) {
      // tensor parallel: all-reduce each expert's fp32 row partials
      for (int idx = tid; idx < p.topk * nb * 16; idx += NC) {
        const int es = idx / (nb * 16), j = (idx / 16) % nb, r = idx % 16;
        const int row = (b0 + j) * 16 + r;
        const float v = row_sum(part + es * nb * BLOCK_PART, j * spb, p.I, r);
        for (int rk = 0; rk < p.tp_world; ++rk)
          tp_slot(rk, p.tp_off_recv_d)[((size_t)p.tp_rank * p.topk + es) * p.H + row] = v;
      }
      sync();
      if (!tp_exchange(p.tp_off_cnt_d, l, b0, b1, OP_DOWN)) return;
      const float* recv = tp_slot(p.tp_rank, p.tp_off_recv_d);
      for (int idx = tid; idx < nb * 16; idx += NC) {
        const int row = b0 * 16 + idx;
        float h = ldcg_bf16(p.hidden + row);
        for (int es = 0; es < p.topk; ++es) {
          float sum = 0.f;
          for (int rk = 0; rk < p.tp_world; ++rk) sum += __ldcg(recv + ((size_t)rk * p.topk + es) * p.H + row);
          h = bf16r(h + bf16r(rscore[es] * bf16r(sum)));
        }
        p.hidden[row] = __float2bfloat16_rn(h);
      }
    } else {
    for (int idx = tid; idx < nb * 16; idx += NC) {
      const int j = idx / 16, r = idx % 16;
      const int row = (b0 + j) * 16 + r;
      float h = ldcg_bf16(p.hidden + row);
      for (int es = 0; es < p.topk; ++es) {
        const float v = bf16r(row_sum(part + es * nb * BLOCK_PART, j * spb, p.I, r));
        h = bf16r(h + bf16r(rscore[es] * v));
      }
      p.hidden[row] = __float2bfloat16_rn(h);
    }
    }
    sync();
    if (tid == 0) red_release_add(bar(l, OP_DOWN - 1, 0), nb * p.topk);
  }

  // Mixtral_RMS_LM_Head (mixtral/python_vm.py:618-642): logits[rows] += bf16
  // partial over one 2048-column split (bf16 atomic add; the caller zeroes
  // logits, and with two splits the sum is independent of their order).
  __device__ void op_lm_head_split(const Ins& ins, const Plan& pl) {
    const int b0 = ins.w[1], b1 = ins.w[2], split = ins.w[3];
    const NormWeights nw = preload_norm(p.lm_norm, p.H);
    {
      int* a = bar(p.L - 1, OP_DOWN - 1, 0);
      const int t = p.down_done_target;
      if (!wait_counters(1, &a, &t, OP_LM_HEAD, p.L - 1)) { drain(pl.ns); return; }
    }
    stamp(TS_READY);
    rmsnorm_to_act(p.hidden, p.lm_norm, p.H, nw);
    stamp(TS_ACT);
    const int spb = stages_per_row_block(LM_HEAD_SPLIT);
    float* part = partials_after(p.H);
    gemv_stream(pl.ns, LM_HEAD_SPLIT, part, split * LM_HEAD_SPLIT);
    stamp(TS_STORE);
    if (p.tp_world > 1) {
      // tensor parallel: this rank's vocabulary rows go into every rank's logits
      for (int idx = tid; idx < (b1 - b0) * 16; idx += NC) {
        const int j = idx / 16, r = idx % 16;
        const __nv_bfloat16 v = __float2bfloat16_rn(row_sum(part, j * spb, LM_HEAD_SPLIT, r));
        const int row = p.lm_row0 + (b0 + j) * 16 + r;
        for (int rk = 0; rk < p.tp_world; ++rk)
          atomicAdd(reinterpret_cast<__nv_bfloat16*>(p.tp_peer[rk] + p.tp_off_logits) + row, v);
      }
      sync();
      if (warp == 0 && lane < p.tp_world) red_release_sys_add(tp_counter(lane, p.tp_off_cnt_lm, 0), 1);
      return;
    }
    for (int idx = tid; idx < (b1 - b0) * 16; idx += NC) {
      const int j = idx / 16, r = idx % 16;
      atomicAdd(p.logits + (b0 + j) * 16 + r, __float2bfloat16_rn(row_sum(part, j * spb, LM_HEAD_SPLIT, r)));
    }
  }

  // SpeculativeExpertPredict (mixtral/python_vm.py:653-668).
  __device__ void op_predict(const Ins& ins) {
    const int l = ins.w[1];
    const NormWeights nw = preload_norm(p.ffn_ln + (size_t)l * p.H, p.H);
    if (l > 0) {
      int* a = bar(l - 1, OP_DOWN - 1, 0);
      const int t = p.down_done_target;
      if (!wait_counters(1, &a, &t, OP_PREDICT, l)) return;
    } else if (!wait_counters(0, nullptr, nullptr, OP_PREDICT, l)) {
      return;
    }
    stamp(TS_READY);
    rmsnorm_to_act(p.hidden, p.ffn_ln + (size_t)l * p.H, p.H, nw);
    router(l);
    if (tid < p.topk) p.pred_idx[tid] = rsel[tid];
    sync();
    if (tid == 0) red_release_add(bar(l, OP_PREDICT - 1, 0), 1);
  }
};

// ------------------------------------------------------------------ loader
// A second walk over the queue's stages, ahead of the loads, issuing L2
// prefetches. It runs only while the ring is full, so the prefetches fill HBM
// idle time (consumers waiting on other SMs) instead of competing with loads.
struct PrefetchCursor {
  int i = 0;
  bool have = false;
  long long g = 0;  // stream index of the walker's current stage
  int issued = 0;   // prefetched stages (diagnostics)
  Ins* ins = nullptr;  // its instruction words (shared memory)
  StageWalker wk;

  // Prefetch (or skip, if already loaded) one stage; false when exhausted.
  __device__ bool step(const KParams& p, int q, long long g_load) {
    while (true) {
      if (!have) {
        if (i >= p.Q) return false;
        fetch_ins(p, q, i, *ins);
        // Mixtral expert instructions: the predicted experts (a hint written
        // by SpeculativeExpertPredict; stale values only cost a wasted prefetch)
        int pred[MAX_TOPK] = {0, 0, 0, 0};
        if (kMixtral)
          for (int t = 0; t < p.topk && t < MAX_TOPK; ++t) pred[t] = ld_relaxed(p.pred_idx + t);
        wk.init(p, *ins, make_plan(p, *ins), pred);
        have = true;
      }
      if (wk.done()) {
        ++i;
        have = false;
        continue;
      }
      if (g >= g_load) {
        wk.issue<true>(p, nullptr, nullptr);
        ++issued;
      } else {
        wk.advance(p);  // already loaded into the ring
      }
      ++g;
      return true;
    }
  }
};

// L2-prefetch the weights of instruction i of queue q: one bulk prefetch per
// contiguous run (per row segment for strided runs), the general walker for
// the rest. KV stages are not prefetched (the partial's range is small and its
// newest rows are written during the step). Mixtral expert instructions use
// the predicted experts (a hint; a wrong guess only wastes the prefetch).
__device__ void prefetch_instruction(const KParams& p, int q, int i, Ins* ins) {
  if (i >= p.Q) return;
  fetch_ins(p, q, i, *ins);
  const Plan pl = make_plan(p, *ins);
  if (pl.bad_word >= 0 || pl.ns == 0 || pl.op == OP_PARTIAL) return;
  int pred[MAX_TOPK] = {0, 0, 0, 0};
  if (kMixtral)
    for (int t = 0; t < p.topk && t < MAX_TOPK; ++t) pred[t] = ld_relaxed(p.pred_idx + t);
  StageWalker w;
  w.init(p, *ins, pl, pred);
  while (!w.done()) {
    StageWalker::Run r;
    const int n = w.contiguous_run(p, r);
    if (n > 0) {
      if (r.chunks > 1) {  // contiguous whole rows in chunks of two sizes
        const uint8_t* src = r.src;
        for (int t = 0; t < n; ++t) {
          const uint32_t sb = (r.c0 + t) % r.chunks == r.chunks - 1 ? r.last_bytes : r.bytes;
          bulk_prefetch_l2(src, sb);
          src += sb;
        }
      } else if (r.copies == 1 && r.stage_step == (long long)r.bytes) {
        bulk_prefetch_l2(r.src, r.bytes * (uint32_t)n);
      } else {
        for (int t = 0; t < n; ++t)
          for (int c = 0; c < r.copies; ++c) bulk_prefetch_l2(r.src + t * r.stage_step + c * r.row_step, r.bytes);
      }
      w.skip_run(p, n);
    } else {
      w.issue<true>(p, nullptr, nullptr);
    }
  }
}

// ------------------------------------------------------------------ MLP prefetcher
// L2 prefetch of [src, src + bytes) by one warp in 16 KiB pieces: per-line
// prefetches through the load/store unit (lane t takes lines t, t + 32, ...),
// or TMA bulk prefetches (PF_BULK); an optional pause after each piece.
__device__ __forceinline__ void warp_prefetch_l2(const KParams& p, const void* src, uint32_t bytes, int lane) {
  const uint8_t* s = static_cast<const uint8_t*>(src);
  constexpr uint32_t PIECE = 16384;
  for (uint32_t o = 0; o < bytes; o += PIECE) {
    const uint32_t n = min(PIECE, bytes - o);
    if (p.pf_mlp & PF_BULK) {
      if (lane == 0) bulk_prefetch_l2(s + o, n);
    } else if (p.pf_mlp & PF_EVICT_LAST) {
      for (uint32_t off = (uint32_t)lane * 128u; off < n; off += 32u * 128u) prefetch_l2_line_last(s + o + off);
    } else {
      for (uint32_t off = (uint32_t)lane * 128u; off < n; off += 32u * 128u) prefetch_l2_line(s + o + off);
    }
    if (p.pf_gap_ns > 0) __nanosleep(p.pf_gap_ns);
  }
}

// The prefetcher warp walks its queue; for each Llama up/gate or down
// instruction of layer l it waits until layer l - 1's down projection is
// complete (from then on the SMs run the attention chain of layer l, whose
// weights are already in the rings) and prefetches the instruction's weight
// rows into L2. Its waits are bounded and it records no errors: on a timeout
// or an aborted launch it simply stops (the consumers report the failure).
__device__ void run_mlp_prefetcher(const KParams& p) {
  const int q = blockIdx.x, lane = threadIdx.x & 31;
  int armed = -1;  // layer whose trigger has been seen
  for (int i = 0; i < p.Q; ++i) {
    const int wv = __ldg(p.instructions + ((size_t)q * p.Q + i) * 32 + lane);  // lane t: word t
    const int op = __shfl_sync(0xffffffffu, wv, 0), l = __shfl_sync(0xffffffffu, wv, 1);
    const bool up = op == OP_UPGATE && (p.pf_mlp & PF_UPGATE);
    const bool dn = op == OP_DOWN && (p.pf_mlp & PF_DOWN);
    if ((!up && !dn) || l < 0 || l >= p.L) continue;
    if (l != armed) {
      if (l > 0) {
        int ok = 1;
        if (lane == 0) {
          const int* c = p.barriers + ((size_t)(l - 1) * p.brow + (OP_DOWN - 1)) * p.bcol;
          const uint64_t t0 = globaltimer();
          while (ld_relaxed(c) < p.down_done_target) {
            if (aborted(p) || (long long)(globaltimer() - t0) > p.timeout_ns) { ok = 0; break; }
            __nanosleep(64);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      }
      armed = l;
    }
    if (up) {
      const int n = __shfl_sync(0xffffffffu, wv, 2);
      if (n < 0 || n > 29) continue;
      for (int j = 0; j < n; ++j) {
        const int b = __shfl_sync(0xffffffffu, wv, 3 + j);
        if (b < 0 || b >= p.I / 16) continue;
        const size_t row = (size_t)l * p.I + (size_t)b * 16;
        warp_prefetch_l2(p, p.w_up + row * p.H, 16u * p.H * 2u, lane);
        warp_prefetch_l2(p, p.w_gate + row * p.H, 16u * p.H * 2u, lane);
      }
    } else {
      const int b0 = __shfl_sync(0xffffffffu, wv, 2), b1 = __shfl_sync(0xffffffffu, wv, 3);
      const int split = __shfl_sync(0xffffffffu, wv, 4);
      if (b0 < 0 || b1 > p.H / 16 || b0 > b1 || split < 0 || split >= p.down_splits) continue;
      for (int r = b0 * 16; r < b1 * 16; ++r)
        warp_prefetch_l2(p, p.w_down + ((size_t)l * p.H + r) * p.I + (size_t)split * p.down_R,
                         (uint32_t)p.down_R * 2u, lane);
    }
  }
}

// Mixtral RmsRouterUpgate: before the loader waits for the router's choice,
// L2-prefetch the first spec_stages ring stages of each predicted expert
// (SpeculativeExpertPredict's output for this layer, awaited with a short
// bound; a late or wrong guess only wastes the prefetch), as the reference's
// loader does (demos/mixtral/rms_router_matvec.cu:258-289).
__device__ void speculative_prefetch(const KParams& p, const Ins& ins, const Plan& pl) {
  const int* c = p.barriers + ((size_t)pl.layer * p.brow + (OP_PREDICT - 1)) * p.bcol;
  const uint64_t t0 = globaltimer();
  while (ld_acquire(c) < 1) {
    if (aborted(p) || (long long)(globaltimer() - t0) > p.timeout_ns) return;
    __nanosleep(64);
  }
  int pred[MAX_TOPK];
  for (int t = 0; t < MAX_TOPK; ++t) pred[t] = t < p.topk ? ld_relaxed(p.pred_idx + t) : 0;
  const int per_expert = min(p.spec_stages, pl.ns / p.topk);
  for (int e = 0; e < p.topk; ++e) {
    int rot[MAX_TOPK];
    for (int t = 0; t < MAX_TOPK; ++t) rot[t] = pred[(e + t) % p.topk];
    StageWalker w;
    w.init(p, ins, pl, rot);
    for (int k = 0; k < per_expert && !w.done(); ++k) w.issue<true>(p, nullptr, nullptr);
  }
}

// lins / pins: shared-memory instruction buffers of the loader and of its L2
// prefetch cursor (dynamically indexed words stay out of local memory).
__device__ void run_loader(const KParams& p, Ring ring, const int* mbox, uint64_t* mbox_bar, Ins* lins,
                           Ins* pins) {
  const int q = blockIdx.x;
  Ins& ins = *lins;
  StageWalker wk;
  PrefetchCursor pf;
  pf.ins = pins;
  int pf_layer = -1;  // layer whose MLP weights were last prefetched (pf_next == 2)
  long long g_load = 0;
  uint32_t mbox_phase = 0;
  const long long ring_timeout = 4 * p.timeout_ns + 2000000000ll;
  const bool ring_ef = (p.pf_mlp & PF_RING_EVICT_FIRST) != 0;
  const uint64_t pol_ef = policy_evict_first();

  for (int i = 0; i < p.Q; ++i) {
    fetch_ins(p, q, i, ins);
    const Plan pl = make_plan(p, ins);
    int ex[MAX_TOPK] = {0, 0, 0, 0};
    if (kMixtral && (pl.op == OP_UPGATE || pl.op == OP_DOWN) && pl.bad_word < 0 && pl.ns > 0) {
      // which experts to stream is decided by the consumers (router, or the
      // router outputs of another SM): wait for their handoff, prefetching
      // ahead into L2 meanwhile
      if (pl.op == OP_UPGATE && p.spec_stages > 0) speculative_prefetch(p, ins, pl);
      while (kPrefetch && p.pf_stages > 0 && pf.g < g_load + p.pf_stages && !mbar_test_wait(mbox_bar, mbox_phase))
        if (!pf.step(p, q, g_load)) break;
      if (!ring_wait(mbox_bar, mbox_phase, ring_timeout)) {
        record_error(p, 4, i, pl.op, pl.layer, -1, (int)mbox_phase, -2);
        return;
      }
      mbox_phase ^= 1u;
      for (int t = 0; t < p.topk && t < MAX_TOPK; ++t) ex[t] = mbox[t];
    }
    wk.init(p, ins, pl, ex);
    if (kPrefetch && p.pf_next == 1) {
      prefetch_instruction(p, q, i + 1, pins);
    } else if (kPrefetch && p.pf_next == 2 && pl.op >= OP_QKV && pl.op <= OP_OPROJ && pl.layer != pf_layer) {
      pf_layer = pl.layer;
      for (int j = i + 1; j < p.Q; ++j) {
        const int* wj = p.instructions + ((size_t)q * p.Q + j) * 32;
        const int opj = __ldg(wj), lj = __ldg(wj + 1);
        if (opj == OP_QKV && lj != pl.layer) break;
        if ((opj == OP_UPGATE || opj == OP_DOWN) && lj == pl.layer) prefetch_instruction(p, q, j, pins);
      }
    }
    while (!wk.done()) {
      StageWalker::Run rr;
      const int run = wk.contiguous_run(p, rr);
      if (run > 0) {  // fast path: stages at a fixed stride
        for (int t = 0; t < run; ++t) {
          uint64_t* empty = &ring.empty[ring.slot];
          const uint32_t parity = ring.phase ^ 1u;
          if (!mbar_test_wait(empty, parity)) {
            bool more = kPrefetch && p.pf_stages > 0;
            while (more && pf.g < g_load + p.pf_stages && !mbar_test_wait(empty, parity))
              more = pf.step(p, q, g_load);
            if (!ring_wait(empty, parity, ring_timeout)) {
              record_error(p, 4, i, pl.op, pl.layer, ring.slot, (int)ring.phase, -1);
              return;
            }
          }
          if (p.record && p.timings && wk.k + t < 16)
            p.timings[((size_t)q * p.Q + i) * 128 + TS_STAGE_LOAD + wk.k + t] = (int)(globaltimer() & 0x7fffffff);
          uint64_t* fb = &ring.full[ring.slot];
          uint8_t* dst = ring.stages + (size_t)ring.slot * STAGE_BYTES;
          const uint32_t sb = (rr.chunks > 1 && (rr.c0 + t) % rr.chunks == rr.chunks - 1) ? rr.last_bytes : rr.bytes;
          mbar_arrive_expect_tx(fb, sb * (uint32_t)rr.copies);
          if (ring_ef)
            for (int c = 0; c < rr.copies; ++c) bulk_load_hint(dst + c * sb, rr.src + c * rr.row_step, sb, fb, pol_ef);
          else
            for (int c = 0; c < rr.copies; ++c) bulk_load(dst + c * sb, rr.src + c * rr.row_step, sb, fb);
          rr.src += rr.chunks > 1 ? (long long)sb : rr.stage_step;
          ring_advance(ring);
          ++g_load;
        }
        wk.skip_run(p, run);
        continue;
      }
      uint64_t* empty = &ring.empty[ring.slot];
      const uint32_t parity = ring.phase ^ 1u;
      if (!mbar_test_wait(empty, parity)) {
        // ring full: run the L2 prefetch ahead while waiting for a slot
        bool more = kPrefetch && p.pf_stages > 0;
        while (more && pf.g < g_load + p.pf_stages && !mbar_test_wait(empty, parity))
          more = pf.step(p, q, g_load);
        if (!ring_wait(empty, parity, ring_timeout)) {
          record_error(p, 4, i, pl.op, pl.layer, ring.slot, (int)ring.phase, -1);
          return;
        }
      }
      if (p.record && p.timings && wk.k < 16)
        p.timings[((size_t)q * p.Q + i) * 128 + TS_STAGE_LOAD + wk.k] = (int)(globaltimer() & 0x7fffffff);
      wk.issue<false>(p, ring.stages + (size_t)ring.slot * STAGE_BYTES, &ring.full[ring.slot]);
      ring_advance(ring);
      ++g_load;
    }
  }
  // diagnostics: stages loaded and prefetched by this queue's loader
  if (p.record && p.timings) {
    p.timings[(size_t)q * p.Q * 128 + TS_DIAG] = pf.issued;
    p.timings[(size_t)q * p.Q * 128 + TS_DIAG + 1] = (int)g_load;
  }
}

}  // namespace

// ------------------------------------------------------------------ kernel
namespace EK_NS {

template <int D>
__global__ void __launch_bounds__(NTHREADS, 1) decode_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  uint8_t* act = smem + NUM_STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(act + ACT_BYTES);
  uint64_t* empty = full + NUM_STAGES;
  uint64_t* mbox_bar = empty + NUM_STAGES;
  float* red = reinterpret_cast<float*>(mbox_bar + 1);
  int* flag = reinterpret_cast<int*>(red + CW);
  int* mbox = flag + 1;                        // MAX_TOPK
  float* rlog = reinterpret_cast<float*>(mbox + MAX_TOPK);  // MAX_EXPERTS
  int* rsel = reinterpret_cast<int*>(rlog + MAX_EXPERTS);   // MAX_TOPK
  float* rscore = reinterpret_cast<float*>(rsel + MAX_TOPK);  // MAX_TOPK
  // instruction words: consumers, loader, loader's prefetch cursor
  Ins* ins_smem = reinterpret_cast<Ins*>(act + ACT_BYTES + 512);
  static_assert(512 + 3 * sizeof(Ins) <= CTRL_BYTES, "control area");

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  if (tid == 0) {
    for (int s = 0; s < NUM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
    mbar_init(mbox_bar, 1);
    fence_mbar_init();
  }
  if (blockIdx.x == 0 && tid == 0 && p.out_token) {  // the next launch's slot (the host may skip one epoch)
    p.status->lm_arrivals[(p.epoch + 1u) & 3u] = 0u;
    p.status->lm_arrivals[(p.epoch + 2u) & 3u] = 0u;
  }
  if (tid == NC) {
    prefetch_tensormap(&p.tm_k);
    prefetch_tensormap(&p.tm_v);
  }
  __syncthreads();

  Ring ring{stages, full, empty, 0, 0u, 0u};
  if (warp == LOADER_WARP) {
    if (lane == 0) run_loader(p, ring, mbox, mbox_bar, ins_smem + 1, ins_smem + 2);
    return;
  }
  if (kPrefetch && warp == PREFETCH_WARP) {
    if ((p.pf_mlp & (PF_UPGATE | PF_DOWN)) && !kMixtral) run_mlp_prefetcher(p);
    return;
  }

  Consumer c(p);
  c.ring = ring;
  c.act = act;
  c.red = red;
  c.flag = flag;
  c.mbox = mbox;
  c.mbox_bar = mbox_bar;
  c.rlog = rlog;
  c.rsel = rsel;
  c.rscore = rscore;
  c.tid = tid;
  c.warp = warp;
  c.lane = lane;
  c.qidx = blockIdx.x;
  c.broken = false;

  Ins& ins = ins_smem[0];
  const int* qwords = p.instructions + (size_t)blockIdx.x * p.Q * 32;
  // instruction words one instruction ahead: warp 0's lane t holds word t of
  // the next instruction, loaded while the current one runs
  int next_word = (tid < 32 && p.Q > 0) ? __ldg(qwords + tid) : 0;
  for (int i = 0; i < p.Q; ++i) {
    c.iidx = i;
    // every consumer finished the previous instruction (trailing barrier)
    if (tid < 32) {
      ins.w[tid] = next_word;
      if (i + 1 < p.Q) next_word = __ldg(qwords + (size_t)(i + 1) * 32 + tid);
    }
    c.sync();
    const Plan pl = make_plan(p, ins);
    c.stamp(TS_START);
    if (pl.bad_word >= 0) {
      if (tid == 0)
        record_error(p, pl.bad_word == 0 && (pl.op < 0 || pl.op > (kMixtral ? OP_PREDICT : OP_LM_HEAD)) ? 2 : 3, i, pl.op,
                     pl.layer, 0, pl.bad_word, ins.w[pl.bad_word]);
      c.sync();  // before the next instruction's words overwrite these
      continue;  // no stages were planned for it
    }
    if (kMixtral && pl.op >= OP_UPGATE) {
      switch (pl.op) {
        case OP_UPGATE: c.op_router_upgate(ins, pl); break;
        case OP_DOWN: c.op_expert_down(ins, pl); break;
        case OP_LM_HEAD: c.op_lm_head_split(ins, pl); break;
        case OP_PREDICT: c.op_predict(ins); break;
        default: break;
      }
      c.stamp(TS_END);
      c.sync();
      continue;
    }
    switch (pl.op) {
      case OP_NOOP: break;
      case OP_QKV: c.op_qkv(ins, pl); break;
      case OP_PARTIAL: c.op_partial<D>(ins, pl); break;
      case OP_REDUCTION: c.op_reduction(ins); break;
      case OP_OPROJ:
      case OP_DOWN: c.op_matvec_add(ins, pl); break;
      case OP_UPGATE: c.op_upgate(ins, pl); break;
      case OP_LM_HEAD: c.op_lm_head(ins, pl); break;
      default: break;
    }
    c.stamp(TS_END);
    c.sync();  // act / red / flag are reused by the next instruction
  }
  // tensor parallel: the logits are complete once every rank's LM-head
  // instructions have added into them; block 0 holds the kernel until then
  if (kMixtral && p.tp_world > 1 && p.tp_lm_count > 0 && blockIdx.x == 0) {
    int* a = c.tp_counter(p.tp_rank, p.tp_off_cnt_lm, 0);
    const int t = p.tp_world * p.tp_lm_count * (int)p.tp_step;
    c.iidx = p.Q;
    c.wait_counters(1, &a, &t, OP_LM_HEAD, p.L - 1, true);
  }
}

// ------------------------------------------------------------------ host launch
cudaError_t launch(const KParams& p, cudaStream_t stream) {
  // The shared-memory opt-in is a per-device function attribute: set it once
  // per (device, head_dim) variant. Devices beyond the table set it on every
  // launch (cheap, and idempotent).
  constexpr int kDevs = 64;
  static std::atomic<unsigned char> attr_done[kDevs][2];
  const void* fn = p.D == 64 ? reinterpret_cast<const void*>(&decode_kernel<64>)
                             : reinterpret_cast<const void*>(&decode_kernel<128>);
  const int which = p.D == 64 ? 0 : 1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kDevs || !attr_done[dev][which].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kDevs) attr_done[dev][which].store(1, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nq);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.D == 64) return cudaLaunchKernelEx(&cfg, decode_kernel<64>, p);
  return cudaLaunchKernelEx(&cfg, decode_kernel<128>, p);
}

}  // namespace EK_NS

}  // namespace ek
