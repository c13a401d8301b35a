// The fused decode step: HIVE Limited's Engine._step() + LM head + greedy argmax
// (engine/limited.py:374-428) as ONE persistent cooperative kernel.
//
// Why one kernel: at batch 1 the step is ~20 dependent launches per layer (the
// reference issues 538 for 28 layers). Each launch boundary drains the GPU; here the
// dependencies become grid barriers inside one launch, and every CTA recomputes the
// small vector work it needs (RMSNorm + per-32 quantisation of a 4-20 KB vector, the
// q/k norms and RoPE of its own heads) instead of waiting on a separate kernel.
//
// Why warp-specialised: the step reads ~6 GB (8B shape at a 4k context) and computes
// little, so its speed is how continuously HBM is kept busy. Each CTA (one per SM) has a
// PRODUCER warp that walks the CTA's share of every byte the step streams -- its weight
// tiles of every GEMV, the K rows of its attention chunk and the V rows and exps of its
// context items, its rows of the LM head
// -- in the order they are consumed, and copies them with the bulk-copy engine
// (cp.async.bulk, completion on an mbarrier) into a ring of 10 KB shared-memory slots.
// Eight CONSUMER warps wait for slots, compute, and release them. Only the consumers
// take part in the grid barriers between phases, so while they wait for the rest of the
// GPU, or build the next activation vector, the producer is already loading the next
// phase's weights (as far as the ring reaches). Nothing the producer streams depends on
// this step's results: weights are constant and the KV rows it reads (positions < pos)
// were written by earlier launches; row `pos` itself comes from this step's qkv output.
//
// Per layer, five phases separated by grid barriers:
//   P1 qkv  : act <- quant(rmsnorm(h, an)); rows of W_qkv        -> qkv
//   P2 attn : A, per (kv head, chunk of numpy's pairwise recursion): q/k norm + RoPE,
//             KV append at pos, scores in OpenBLAS's order, exps and the chunk's
//             subtree sum; B, per (query head, 32-dim slice), once its kv head's chunks
//             are in: the sequential weighted V sum               -> ctx
//   P3 o    : act <- quant(ctx);   rows of W_o, h[row] += y        -> h
//   P4 gu   : act <- quant(rmsnorm(h, fn)); gate/up row pairs, SiLU -> act
//   P5 down : act <- quant(act);   rows of W_down, h[row] += y     -> h
// then the head: act <- quant(rmsnorm(h, onorm)); rows of the LM head -> logits and a
// per-CTA argmax; the last CTA picks the token and advances tok/gen/step/pos.
//
// GEMV tiles split evenly over the CTAs; the CTAs that take the remainder's extra tile
// rotate from phase to phase. Data produced by other CTAs is read through L2
// (ld.global.cg) after a grid barrier: L1 is not coherent across SMs.
#include <mutex>

#include <cuda.h>
#include <cuda_fp16.h>

#include "attn_exact.cuh"
#include "gemv_mma.cuh"
#include "hv_internal.h"
#include "hv_wait.cuh"

namespace hv {

constexpr int kConsWarps = 8;                          // consumer warps
constexpr int kConsThreads = kConsWarps * 32;
constexpr int kStepThreads = kConsThreads + 32;        // + the producer warp
constexpr int kSlotBytes = 10240;                      // one ring slot
constexpr int kSlotIters = 8;                          // GEMV iterations per slot
constexpr int kSlotScaleOff = kSlotIters * kPpNibWords * 4;   // nibbles, then scales
constexpr int kSlotRows = kSlotBytes / (kHd * 4);      // KV rows per slot (20)
constexpr int kMaxSlots = 32;
constexpr int kMaxHidden = 8192;                       // pro_norm_quant's registers
constexpr int kSmemLimit = 227 * 1024;
constexpr unsigned long long kWaitNs = 2000000000ull;          // consumer waits: 2 s
constexpr unsigned long long kProducerWaitNs = 4000000000ull;  // producer waits: 4 s

static_assert(kSlotScaleOff + kSlotIters * kPpScales * 4 == kSlotBytes, "slot layout");
static_assert(sizeof(hv_layer_w) % 8 == 0, "layer table copied as 8-byte words");
static_assert(kSlotRows % 4 == 0, "attention groups of 4 rows never straddle slots");
static_assert(kSlotRows == kAttnBlock, "a ring slot of KV rows is one attention block");

// Phase B (the context) runs one item per (query head, 32-dim slice): a chain warp adds
// the products w_t v_t[d] of its 32 dims position after position, while helper warps of
// the same CTA form those products from the ring's V rows and the head's exps and hand
// them over transposed, so that the chain reads four positions per 16-byte load. Block u
// (counted over the launch) goes to helper u % 4 and its products buffer.
constexpr int kCtxRows = 64;                           // V rows per phase-B slot (a block)
constexpr int kCtxHelpers = 4;                         // helper warps: 1, 2, 3 and 5
constexpr int kCtxPStride = kCtxRows + 4;              // floats per dim in a products buffer
constexpr int kCtxPBufs = kCtxHelpers;                 // one products buffer per helper
constexpr int kCtxPFloats = 32 * kCtxPStride;          // one products buffer
static_assert(kCtxPBufs == 4, "StepShared holds four products-buffer barrier pairs");
static_assert(kCtxRows * (32 * 4 + 4) <= kSlotBytes, "a phase-B slot: V rows + exps");
static_assert(kCtxRows == 64, "a helper divides two rows per lane");
static_assert((kCtxPStride / 4) % 2 == 1, "products buffer: conflict-free 16-byte accesses");


// Run-time tunables (hv_step_set_option): bulk copies a producer keeps in flight, and
// whether streamed bytes are marked evict-first in L2. Copies beyond what saturates HBM
// only queue in front of the consumers' own (latency-critical) loads.
static int g_opt_inflight = 6;
static int g_opt_evict_first = 1;
static int g_opt_local_qkv_barrier = 0;
// Launch flag set by the library (not by callers): the barrier after the qkv projection
// of a sharded step stays among the rank's own CTAs.
constexpr int kFlagLocalQkvBarrier = 1 << 8;

using CSync = SyncNamed<kConsThreads, 1>;
HV_DEV void csync() { CSync::sync(); }

// Reduction plans of the step, built on the host (hv_step_plans) and copied into shared
// memory at the start of every launch.
struct StepPlans {
  PwPlan pw_hid;                 // RMSNorm over the hidden vector
  GvPlan gv_hid, gv_o, gv_ffn;   // GEMV rows with K = hidden, n_head * 128, ffn
};

struct StepShared {
  StepPlans P;
  float leafval[kPwMaxLeaf];
  float red[4];
  float sv[32];
  int si[32];
  int flag;
  int ok;
  int abort;                     // set by any warp of this CTA whose wait gave up
  int tree_ok;                   // the pairwise tree of the softmax sum was built
  BlasRuns runs;                 // the reference host's gemv runs over pos + 1 rows
  PwFront front;                 // the attention chunks: numpy's recursion cut at a depth
  unsigned phase;                // top bit of the grid barrier counter to wait for next
  unsigned xphase;               // sharded: top bit of the cross-rank counter (CTA 0)
  unsigned gen;                  // sharded: generation of the local release word
  unsigned long long wait[kConsWarps];   // ns each consumer warp waited for ring slots
  long long busy[kConsWarps];            // cycles spent computing attention scores
  unsigned long long ctx_wait_ns;        // phase B, whole launch: ns the chain waited for products
  unsigned long long ctx_sum_ns;         // phase B, whole launch: ns helper 0 waited for V slots
  uint64_t pfull[4];             // phase B: products buffer b written (its helper arrives)
  uint64_t pfree[4];             // phase B: products buffer b read by the chain (one arrive)
  unsigned pseq;                 // phase B: products buffers used so far in this launch
};

// Byte offsets of the dynamic shared memory regions (host and device agree).
struct StepLayout {
  size_t layers, bars, act_q, act_sb, tree, work, ring, total;
};

HV_HD size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Floats of the attention work area: phase A (q rows, this step's k and v rows, the
// norm scratch, the chunk's scores, the chunk's pairwise tree per head) or phase B (the
// chunks' sums, S, two products buffers, the helpers' weights), whichever is larger.
HV_HD size_t attn_area_floats(int gs, int cap, int nch) {
  const size_t cm = (size_t)front_chunk_max(cap, nch);
  const size_t nvl = ((size_t)pw_tree_nodes_max((int)cm) + 3) & ~size_t(3);
  const size_t a = (size_t)gs * kHd + 2 * kHd + (size_t)(gs + 1) * kHd + 8 +
                   ((cm * gs + 3) & ~size_t(3)) + (size_t)gs * nvl;
  const size_t b = (((size_t)nch + 3) & ~size_t(3)) + 4 + (size_t)kCtxPBufs * kCtxPFloats +
                   (size_t)kCtxHelpers * kCtxRows;
  return a > b ? a : b;
}

HV_HD StepLayout step_layout(int gs, int hid, int qdim, int ffn, int cap, int nch, int nslots,
                             int n_layer) {
  const int kmax = hid > qdim ? (hid > ffn ? hid : ffn) : (qdim > ffn ? qdim : ffn);
  StepLayout L;
  L.layers = align_up(sizeof(StepShared), 16);
  L.bars = L.layers + align_up((size_t)n_layer * sizeof(hv_layer_w), 16);
  L.act_q = L.bars + 2 * kMaxSlots * sizeof(uint64_t);
  L.act_sb = L.act_q + align_up((size_t)kmax, 16);
  L.tree = L.act_sb + align_up((size_t)(kmax / kBlock) * 8, 16);
  L.work = L.tree + align_up(sizeof(PwTree), 16);
  const size_t attn = attn_area_floats(gs, cap, nch) * 4;
  const size_t norm = (size_t)hid * 4;
  L.ring = align_up(L.work + (attn > norm ? attn : norm), 128);
  L.total = L.ring + (size_t)nslots * kSlotBytes;
  return L;
}

// ---- mbarriers and bulk copies -----------------------------------------------------------

HV_DEV unsigned sm_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

HV_DEV void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(sm_addr(b)), "r"(count) : "memory");
}
HV_DEV void mbar_arrive_tx(uint64_t* b, unsigned bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\t"
               "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               :: "r"(sm_addr(b)), "r"(bytes) : "memory");
}
HV_DEV void mbar_arrive_n(uint64_t* b, unsigned n) {
  asm volatile("{\n\t.reg .b64 st;\n\t"
               "mbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}"
               :: "r"(sm_addr(b)), "r"(n) : "memory");
}
HV_DEV bool mbar_test(uint64_t* b, unsigned parity) {
  unsigned ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(sm_addr(b)), "r"(parity) : "memory");
  return ok != 0;
}
// Non-blocking test (try_wait may suspend the thread for a while before failing).
HV_DEV bool mbar_probe(uint64_t* b, unsigned parity) {
  unsigned ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(sm_addr(b)), "r"(parity) : "memory");
  return ok != 0;
}
// The same test, but a thread whose phase has not completed is suspended (up to
// hint_ns) until it does, instead of spinning on the issue slots other warps need.
HV_DEV bool mbar_test_sleep(uint64_t* b, unsigned parity, unsigned hint_ns) {
  unsigned ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(sm_addr(b)), "r"(parity), "r"(hint_ns) : "memory");
  return ok != 0;
}
// global -> this CTA's shared memory, `bytes` (multiple of 16, both addresses 16-byte
// aligned), completion counted on mbarrier `bar`
HV_DEV void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(sm_addr(dst)), "l"(src), "r"(bytes), "r"(sm_addr(bar)) : "memory");
}
// the same with an L2 cache policy (createpolicy)
HV_DEV void bulk_load_hint(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                           unsigned long long policy) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
               " [%0], [%1], %2, [%3], %4;"
               :: "r"(sm_addr(dst)), "l"(src), "r"(bytes), "r"(sm_addr(bar)), "l"(policy)
               : "memory");
}
HV_DEV unsigned long long policy_evict_first() {
  unsigned long long p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}


// Bounded wait for the completion of phase `parity` of mbarrier b. Gives up (false) when
// this CTA has aborted, when any CTA reported a failure in *status, or after `limit` ns
// (then records HV_E_TIMEOUT). Every caller that gives up sets S.abort.
HV_DEV bool mbar_wait(uint64_t* b, unsigned parity, StepShared& S, int* status,
                      unsigned long long limit) {
  if (mbar_test(b, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned n = 0;; ++n) {
    if (mbar_test_sleep(b, parity, 20000u)) return true;
    if (*(volatile int*)&S.abort) return false;
    if ((n & 7) == 7 && *(volatile int*)status != 0) break;
    if (global_ns() - t0 > limit) {
      atomicCAS(status, 0, HV_E_TIMEOUT);
      break;
    }
  }
  *(volatile int*)&S.abort = 1;
  return false;
}

// A warp's wait: every lane waits; the warp goes on only if all lanes saw the phase.
// The time a warp spends waiting for slots is added to S.wait[warp] (for the trace).
HV_DEV bool warp_wait(uint64_t* b, unsigned parity, StepShared& S, int* status) {
  if (__all_sync(0xFFFFFFFFu, mbar_probe(b, parity))) return true;
  const unsigned long long t0 = global_ns();
  const bool ok = mbar_wait(b, parity, S, status, kWaitNs);
  if ((threadIdx.x & 31) == 0) S.wait[threadIdx.x >> 5] += global_ns() - t0;
  return __all_sync(0xFFFFFFFFu, ok);
}

// The slot ring. Sequence number q (counted identically by producer and consumers) maps
// to slot q % ns; its full barrier completes phase q / ns when the data has landed, its
// empty barrier (kConsWarps arrivals) when the consumers are done with it.
struct Ring {
  unsigned char* slots;
  uint64_t* full;
  uint64_t* empty;
  int ns;
  HV_DEV unsigned char* slot(unsigned q) const { return slots + (size_t)(q % ns) * kSlotBytes; }
  HV_DEV uint64_t* full_of(unsigned q) const { return full + q % ns; }
  HV_DEV uint64_t* empty_of(unsigned q) const { return empty + q % ns; }
  HV_DEV unsigned parity(unsigned q) const { return (q / ns) & 1u; }
};

// Bounded poll of a barrier word until (value & mask) == want; false (HV_E_TIMEOUT, or
// another failure already reported on this rank) when it gives up.
template <bool kSys>
HV_DEV bool poll_word(const unsigned* w, unsigned mask, unsigned want, int* status) {
  return poll_word_until<kSys>(w, mask, want, status, kWaitNs);
}

// Grid-wide barrier of the consumer threads over self-resetting counters: the first
// arrival adds 2^31 - (n - 1), the n - 1 others add 1, so the top bit flips exactly when
// all n have arrived and the low bits return to zero. Each CTA knows which top bit to
// wait for (read once per launch, flipped at every barrier), so arriving is a
// fire-and-forget release add and waiting is one acquire load per poll.
// Sharded step (world > 1), two levels: the rank's CTAs meet on its local counter
// (barrier[0]); the rank's CTA 0 then meets the other ranks' CTA 0 on the cross-rank
// counter (barrier[1] of every rank, NVLink atomics: `world` per barrier, not one per
// CTA), and releases its CTAs by advancing the generation word barrier[2]. Every CTA
// fences its peer stores at system scope before it arrives. Waits are bounded (kWaitNs,
// or until a failure is reported on this rank, or this CTA aborted): the failure is
// recorded and every consumer thread gets false.
// `cross` false: a sharded step's barrier among this rank's CTAs only, for a phase whose
// consumers read nothing the other ranks wrote (attention after the qkv projection: each
// rank owns its heads).
HV_DEV bool grid_sync(const hv_step_desc& D, StepShared& S, bool cross = true) {
  csync();
  if (threadIdx.x == 0) {
    int ok = *(volatile int*)&S.abort == 0;
    if (ok) {
      const unsigned add = (blockIdx.x == 0) ? (0x80000000u - (gridDim.x - 1)) : 1u;
      const unsigned want = S.phase ^ 0x80000000u;
      if (D.world <= 1 || !cross) {
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(D.barrier), "r"(add)
                     : "memory");
        ok = poll_word<false>(D.barrier, 0x80000000u, want, D.status);
      } else {
        __threadfence_system();     // this CTA's peer stores before its arrival
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(D.barrier), "r"(add)
                     : "memory");
        const unsigned gen = S.gen + 1;
        if (blockIdx.x == 0) {
          ok = poll_word<false>(D.barrier, 0x80000000u, want, D.status);
          if (ok) {
            const unsigned xadd = D.rank == 0 ? 0x80000000u - (D.world - 1) : 1u;
            const unsigned xwant = S.xphase ^ 0x80000000u;
            __threadfence_system();
            for (int k = 0; k < D.world; ++k)
              asm volatile("red.release.sys.global.add.u32 [%0], %1;"
                           :: "l"(D.peers->barrier[k] + 1), "r"(xadd) : "memory");
            ok = poll_word<true>(D.barrier + 1, 0x80000000u, xwant, D.status);
            S.xphase = xwant;
            if (ok)
              asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(D.barrier + 2), "r"(gen)
                           : "memory");
          }
        } else {
          ok = poll_word<false>(D.barrier + 2, 0xFFFFFFFFu, gen, D.status);
        }
        S.gen = gen;
      }
      S.phase = want;
    }
    if (!ok) *(volatile int*)&S.abort = 1;
    S.ok = ok;
  }
  csync();
  return S.ok != 0;
}

// Trace entry idx <- the ns warp 0 waited for slots since the last call; restarts the count.
HV_DEV void trace_wait(const hv_step_desc& D, StepShared& S, int idx) {
  if (threadIdx.x == 0) {
    if (D.trace != nullptr)
      D.trace[(size_t)blockIdx.x * HV_STEP_TRACE_STRIDE(D.n_layer) + idx] = S.wait[0];
    S.wait[0] = 0;
  }
}

HV_DEV void trace_mark(const hv_step_desc& D, int idx) {
  if (D.trace != nullptr && threadIdx.x == 0)
    D.trace[(size_t)blockIdx.x * HV_STEP_TRACE_STRIDE(D.n_layer) + idx] = global_ns();
}

// ---- the schedule (walked identically by the producer and the consumers) --------------

// Tiles [t0, t1) of a GEMV phase for this CTA: ntiles / grid each, and one more for the
// `extra` CTAs starting at *off (cyclically). *off advances by extra, so the remainder
// moves on to other CTAs in the next phase.
HV_DEV void phase_tiles(int ntiles, int* off, int* t0, int* t1) {
  const int G = gridDim.x, s = blockIdx.x;
  const int base = ntiles / G, extra = ntiles % G, o = *off;
  const int e1 = min(o + extra, G), wrap = max(0, o + extra - G);
  const int b0 = max(0, min(s, e1) - o) + min(s, wrap);
  const int b1 = max(0, min(s + 1, e1) - o) + min(s + 1, wrap);
  *t0 = s * base + b0;
  *t1 = (s + 1) * base + b1;
  *off = (o + extra) % G;
}

// Tiles [t0, t1) of the gate/up phase: whole units of 8 tiles (= 32 SiLU outputs, one
// quantisation block), so each CTA quantises the blocks it produced.
HV_DEV void gu_tiles(int ffn, int* off, int* t0, int* t1) {
  const int ntiles = pp_tiles(2 * ffn, ffn);
  int u0, u1;
  phase_tiles((ntiles + 7) / 8, off, &u0, &u1);
  *t0 = min(u0 * 8, ntiles);
  *t1 = min(u1 * 8, ntiles);
}

HV_DEV int slots_per_tile(int niter) { return (niter + kSlotIters - 1) / kSlotIters; }

// Ring sequence number (relative to the phase's first) of slot j of local tile lt. Rows
// of one pairwise leaf (one work item per tile, tile i to warp i % 8) are filled in
// waves: slot 0 of tiles 8R .. 8R+7, then their slot 1, ..., the order the eight warps
// consume them, so free slots go to real prefetch instead of to each warp's later slots.
// Rows of several leaves (items share slots) keep tile-major order.
HV_DEV unsigned slot_seq(int lt, int j, int ntile, int spt, bool wave) {
  if (!wave) return (unsigned)(lt * spt + j);
  const int r = lt / kConsWarps, nr = min(kConsWarps, ntile - r * kConsWarps);
  return (unsigned)(r * kConsWarps * spt + j * nr + (lt - r * kConsWarps));
}

// L2 prefetch (one thread) of a layer's small vectors a phase before they are needed:
// the input norm and the q/k norms (attn) or the post-attention norm. The weights and
// KV rows go through the ring; these few KB would otherwise be demand misses on the
// critical path.
HV_DEV void prefetch_vectors(const hv_layer_w* L, int hid, bool attn) {
  if (attn) {
    prefetch_l2(L->an, (size_t)hid * 4);
    prefetch_l2(L->qn, kHd * 4);
    prefetch_l2(L->kn, kHd * 4);
  } else {
    prefetch_l2(L->fn, (size_t)hid * 4);
  }
}


// Helper index of consumer warp w (warps 1, 2, 3, 5: SM sub-partitions 1-3, none beside
// the chain warp 0), or -1.
HV_DEV int ctx_helper(int w) { return w >= 1 && w <= 3 ? w - 1 : w == 5 ? 3 : -1; }

// The j-th phase-B item of CTA b, or -1. Up to one item per CTA the items spread over the
// grid; past that CTA b takes items b, b + grid, b + 2 grid, ...
HV_DEV int ctx_item(int b, int grid, int nitems, int j) {
  if (nitems > grid) {
    const long long k = (long long)j * grid + b;
    return k < nitems ? (int)k : -1;
  }
  if (j > 0) return -1;
  const int k = (int)(((long long)b * nitems + grid - 1) / grid);
  return (k < nitems && (int)(((long long)k * grid) / nitems) == b) ? k : -1;
}

// Rows [t0, t1) of chunk c of the launch's frontier (empty past its last chunk), and te:
// rows [t0, te) come from the cache, row pos (if in the chunk) from this step's qkv.
HV_DEV void front_rows(const PwFront& F, int pos, int c, int* t0, int* t1, int* te) {
  if (c < F.n) {
    *t0 = F.cb[c];
    *t1 = F.cb[c + 1];
  } else {
    *t0 = *t1 = pos + 1;
  }
  *te = max(*t0, min(*t1, pos));
}

// The attention scratch of the fused step (hv_step_desc.part): per query head the
// chunks' maxima and pairwise sums [n_head][chunks], then the exps [n_head][ew] (ew = cap
// rounded up to 4, rows 16-byte aligned) and room for one block past the last row.
struct StepScratch {
  float* cmax;
  float* nsum;
  float* exps;
  int ew;
};
HV_HD size_t step_part_floats(int nq, int cap, int nch) {
  const size_t a = ((size_t)nq * nch + 3) & ~size_t(3);
  return 2 * a + (size_t)nq * (((size_t)cap + 3) & ~size_t(3)) + 256;
}
HV_DEV StepScratch step_scratch(const hv_step_desc& D) {
  const size_t a = ((size_t)D.n_head * D.attn_chunks + 3) & ~size_t(3);
  return StepScratch{D.part, D.part + a, D.part + 2 * a, (D.cap + 3) & ~3};
}

// One thread: bounded wait until *w >= want (acquire); false (and HV_E_TIMEOUT, unless a
// failure is already recorded) when it gives up.
HV_DEV bool wait_count(const int32_t* w, unsigned want, int* status) {
  const unsigned* p = reinterpret_cast<const unsigned*>(w);
  if (ld_acquire(p) >= want) return true;
  const unsigned long long t0 = global_ns();
  while (ld_acquire(p) < want) {
    if (*(volatile int*)status != 0) return false;
    if (global_ns() - t0 > kWaitNs) {
      atomicCAS(status, 0, HV_E_TIMEOUT);
      return false;
    }
    __nanosleep(100);
  }
  return true;
}

// ---- the producer ----------------------------------------------------------------------

struct Producer {
  const Ring& R;
  StepShared& S;
  int* status;
  unsigned inflight;             // copies allowed in flight (<= ring slots)
  bool hint;
  unsigned long long policy;
  unsigned q = 0;
  bool live = true;
  unsigned long long t_empty = 0, t_flight = 0;   // ns blocked on free slots / on copies

  HV_DEV Producer(const Ring& r, StepShared& s, int* st, int infl, int evict_first)
      : R(r), S(s), status(st) {
    inflight = (unsigned)max(1, min(infl, r.ns));
    hint = evict_first != 0;
    policy = hint ? policy_evict_first() : 0ull;
  }

  // Waits until the next slot's previous contents were released and (cap) until fewer
  // than `inflight` earlier copies are still in flight; false if the wait gave up.
  HV_DEV bool claim(bool cap = true) {
    if (!live) return false;
    if (q >= (unsigned)R.ns && !mbar_probe(R.empty_of(q), R.parity(q) ^ 1u)) {
      const unsigned long long t0 = global_ns();
      if (!mbar_wait(R.empty_of(q), R.parity(q) ^ 1u, S, status, kProducerWaitNs)) {
        live = false;
        return false;
      }
      t_empty += global_ns() - t0;
    }
    if (cap && q >= inflight) {
      const unsigned p = q - inflight;
      if (!mbar_probe(R.full_of(p), R.parity(p))) {
        const unsigned long long t0 = global_ns();
        if (!mbar_wait(R.full_of(p), R.parity(p), S, status, kProducerWaitNs)) {
          live = false;
          return false;
        }
        t_flight += global_ns() - t0;
      }
    }
    return true;
  }

  // Claims the next slot and starts up to two bulk copies into it.
  HV_DEV void issue(const void* a, unsigned na, const void* b, unsigned nb_, unsigned b_off) {
    if (!claim()) return;
    unsigned char* dst = R.slot(q);
    uint64_t* full = R.full_of(q);
    mbar_arrive_tx(full, na + nb_);
    if (hint) {
      bulk_load_hint(dst, a, na, full, policy);
      if (nb_) bulk_load_hint(dst + b_off, b, nb_, full, policy);
    } else {
      bulk_load(dst, a, na, full);
      if (nb_) bulk_load(dst + b_off, b, nb_, full);
    }
    ++q;
  }

  // This CTA's tiles [t0, t1) of a prepacked matrix with niter iterations per tile.
  HV_DEV void gemv_slot(const uint32_t* pb4, const float* psw, int niter, int tile, int j) {
    const int it0 = j * kSlotIters;
    const unsigned n = (unsigned)min(kSlotIters, niter - it0);
    const size_t first = (size_t)tile * niter + it0;
    issue(pb4 + first * kPpNibWords, n * kPpNibWords * 4, psw + first * kPpScales,
          n * kPpScales * 4, kSlotScaleOff);
  }

  // This CTA's tiles [t0, t1) of a prepacked matrix with niter iterations per tile, in the
  // order of slot_seq.
  HV_DEV void gemv(const uint32_t* pb4, const float* psw, int niter, int t0, int t1, int nleaf) {
    const int spt = slots_per_tile(niter), ntile = t1 - t0;
    if (nleaf > 1) {
      for (int lt = 0; lt < ntile && live; ++lt)
        for (int j = 0; j < spt; ++j) gemv_slot(pb4, psw, niter, t0 + lt, j);
      return;
    }
    for (int r0 = 0; r0 < ntile && live; r0 += kConsWarps) {
      const int nr = min(kConsWarps, ntile - r0);
      for (int j = 0; j < spt; ++j)
        for (int i = 0; i < nr; ++i) gemv_slot(pb4, psw, niter, t0 + r0 + i, j);
    }
  }

  // K rows [t0, te) of kv head g for one attention work item (KT: the cache's element
  // type, float or __half), kSlotRows rows per slot.
  template <class KT>
  HV_DEV void krows(const KT* kc, int g, int cap, int t0, int te) {
    const KT* base = kc + (size_t)g * cap * kHd;
    for (int r = t0; r < te && live; r += kSlotRows) {
      const unsigned n = (unsigned)min(kSlotRows, te - r);
      issue(base + (size_t)r * kHd, n * kHd * (unsigned)sizeof(KT), nullptr, 0, 0);
    }
  }

  // The slot's V part: the 32-dim slice x0 .. x0 + 31 of BR rows from row y0 of the
  // cache's 2-D view `vmap` (a tensor copy; rows past the view read zeros). Completes on
  // the slot's full barrier, which expects `total` bytes (the exps come later).
  HV_DEV void vpart(const CUtensorMap* vmap, int x0, int y0, unsigned total) {
    unsigned char* dst = R.slot(q);
    uint64_t* full = R.full_of(q);
    mbar_arrive_tx(full, total);
    if (hint)
      asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
                   " [%0], [%1, {%2, %3}], [%4], %5;"
                   :: "r"(sm_addr(dst)), "l"(vmap), "r"(x0), "r"(y0), "r"(sm_addr(full)),
                      "l"(policy) : "memory");
    else
      asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                   " [%0], [%1, {%2, %3}], [%4];"
                   :: "r"(sm_addr(dst)), "l"(vmap), "r"(x0), "r"(y0), "r"(sm_addr(full))
                   : "memory");
  }

  // The slot of sequence number qs gets its exps part: `bytes` from e0, at byte voff.
  HV_DEV void epart(unsigned qs, const float* e0, unsigned bytes, unsigned voff) {
    unsigned char* dst = R.slot(qs) + voff;
    uint64_t* full = R.full_of(qs);
    if (hint) bulk_load_hint(dst, e0, bytes, full, policy);
    else bulk_load(dst, e0, bytes, full);
  }

  // Non-blocking claim: true if the next slot is free (and, cap, the in-flight limit
  // allows a copy now).
  HV_DEV bool try_claim(bool cap = true) {
    if (!live) return false;
    if (q >= (unsigned)R.ns && !mbar_probe(R.empty_of(q), R.parity(q) ^ 1u)) return false;
    if (cap && q >= inflight && !mbar_probe(R.full_of(q - inflight), R.parity(q - inflight)))
      return false;
    return true;
  }

  // The phase-B slots of one item (a query head and a 32-dim slice x0 .. x0 + 31 of its kv
  // head's V rows from row y0): per block k < nblk, kCtxRows V rows and the head's exps
  // e0 + k kCtxRows .... V parts of the first blocks go out while slots are free without
  // waiting; the exps only once every chunk of the kv head has written them (the second
  // ticket `tk` reaches `want`). The chain consumes a slot in a few hundred cycles, far
  // less than a copy's latency, so these copies take the whole ring (no in-flight cap).
  template <class KT>
  HV_DEV void ctx_slots(const CUtensorMap* vmap, int x0, int y0, const float* e0, int nblk,
                        const int32_t* tk, unsigned want) {
    constexpr unsigned kVB = kCtxRows * 32 * sizeof(KT), kEB = kCtxRows * 4;
    const unsigned qb = q;
    int k = 0;
    for (; k < nblk && try_claim(false); ++k, ++q) vpart(vmap, x0, y0 + k * kCtxRows, kVB + kEB);
    if (!live) return;
    if (!wait_count(tk, want, status)) {
      live = false;
      return;
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");   // exps written by other SMs
    for (int kk = 0; kk < k; ++kk) epart(qb + kk, e0 + (size_t)kk * kCtxRows, kEB, kVB);
    for (; k < nblk && live; ++k) {
      if (!claim(false)) return;
      vpart(vmap, x0, y0 + k * kCtxRows, kVB + kEB);
      epart(q, e0 + (size_t)k * kCtxRows, kEB, kVB);
      ++q;
    }
  }
};

// Wait (bounded) until every copy this producer started has landed, so no bulk copy is
// still writing into shared memory when the CTA exits (on an abort the consumers may
// leave without waiting for their slots).
HV_DEV void producer_drain(const Ring& R, unsigned q, StepShared& S) {
  const unsigned first = q > (unsigned)R.ns ? q - R.ns : 0u;
  const unsigned long long t0 = global_ns();
  for (unsigned k = first; k < q; ++k)
    while (!mbar_test(R.full_of(k), R.parity(k)) && global_ns() - t0 < kWaitNs) {
    }
}

template <int GS, class KT>
HV_DEV void produce(const hv_step_desc& D, const hv_layer_w* Ls, int flags, int pos,
                    const Ring& R, StepShared& S, int inflight, int evict_first,
                    const CUtensorMap* vmap) {
  Producer P(R, S, D.status, inflight, evict_first);
  const int world = D.world > 1 ? D.world : 1;
  const int hid = D.hidden, ffn = D.ffn, qdim = D.n_head * kHd * world, hrows = hid / world;
  const int nqkv = (D.n_head + 2 * D.n_kv) * kHd;
  const int nch = D.attn_chunks;
  const int it_hid = pp_iters(hid / kBlock), it_q = pp_iters(qdim / kBlock),
            it_ffn = pp_iters(ffn * world / kBlock);
  const int nitems = D.n_head * kSlices;
  const long long rowb = (long long)kHd * sizeof(KT);
  int off = 0, t0, t1;
  for (int l = 0; l < D.n_layer && P.live; ++l) {
    const hv_layer_w* L = Ls + l;
    phase_tiles(pp_tiles(nqkv, 0), &off, &t0, &t1);
    P.gemv(L->qkv_b4, L->qkv_sw, it_hid, t0, t1, S.P.gv_hid.nleaf);
    if ((int)blockIdx.x < D.n_kv * nch) {            // this CTA's chunk: K rows
      int a0, a1, ae;
      front_rows(S.front, pos, blockIdx.x % nch, &a0, &a1, &ae);
      P.krows(reinterpret_cast<const KT*>(L->kc), blockIdx.x / nch, D.cap, a0, ae);
    }
    for (int j = 0; P.live; ++j) {                   // this CTA's context items
      const int item = ctx_item(blockIdx.x, gridDim.x, nitems, j);
      if (item < 0) break;
      const int h = item / kSlices, g = h / GS;
      const long long vrow = ((const char*)L->vc - (const char*)D.kv_base) / rowb +
                             (long long)g * D.cap;
      const StepScratch X = step_scratch(D);
      P.ctx_slots<KT>(vmap, 32 * (item % kSlices), (int)vrow, X.exps + (size_t)h * X.ew,
                      (pos + kCtxRows) / kCtxRows, D.ticket + D.n_kv + g,
                      (unsigned)((l + 1) * nch));
    }
    phase_tiles(pp_tiles(hrows, 0), &off, &t0, &t1);
    P.gemv(L->o_b4, L->o_sw, it_q, t0, t1, S.P.gv_o.nleaf);
    gu_tiles(ffn, &off, &t0, &t1);
    P.gemv(L->gu_b4, L->gu_sw, it_hid, t0, t1, S.P.gv_hid.nleaf);
    phase_tiles(pp_tiles(hrows, 0), &off, &t0, &t1);
    P.gemv(L->dn_b4, L->dn_sw, it_ffn, t0, t1, S.P.gv_ffn.nleaf);
  }
  if ((flags & HV_STEP_HEAD) && P.live) {
    phase_tiles(pp_tiles(D.head_rows, 0), &off, &t0, &t1);
    P.gemv(D.head_b4, D.head_sw, it_hid, t0, t1, S.P.gv_hid.nleaf);
  }
  producer_drain(R, P.q, S);
  if (D.trace != nullptr) {
    uint64_t* tr = D.trace + (size_t)blockIdx.x * HV_STEP_TRACE_STRIDE(D.n_layer) + 2 +
                   28 * D.n_layer;
    tr[3] = P.t_empty;
    tr[4] = P.t_flight;
    tr[5] = P.q;
    tr[6] = S.ctx_wait_ns;      // the consumers' phase-B totals (they finished before the
    tr[7] = S.ctx_sum_ns;       // producer's drain returned: every slot was released)
  }
}

// ---- prologues: build the quantised activation in shared memory ---------------------

// One float4 of a vector, quantised by its 8-lane group (one 32-block): optionally
// normalised first (w * (x / d)). Out of line so that the division-heavy code exists
// once, not once per unrolled load: the prologues run once per phase, with an
// instruction cache that the phase in between has refilled.
__device__ __noinline__ unsigned quant4(float4 x, float4 w, float d, bool norm, int b,
                                        bool lead, int2* sb_s) {
  if (norm)
    x = make_float4(__fmul_rn(w.x, __fdiv_rn(x.x, d)), __fmul_rn(w.y, __fdiv_rn(x.y, d)),
                    __fmul_rn(w.z, __fdiv_rn(x.z, d)), __fmul_rn(w.w, __fdiv_rn(x.w, d)));
  float s;
  int bs;
  const unsigned q = quant_block_8lanes(x, &s, &bs);
  if (lead) sb_s[b] = make_int2(__float_as_int(s), bs);
  return q;
}

// act <- quant(rmsnorm(src, w)) over n = hidden values (n % 32 == 0,
// n <= KV * 4 * kConsThreads); src from global (through L2) or, for layer 0, the f16
// embedding row. Thread t holds float4 i4 = t + 256 k, so the 8 lanes of a lane group
// hold one 32-block and quantise it from registers. KV (float4 per thread) is a template
// argument so the normalise/quantise chains of a thread's blocks are inline and
// interleave, with code for exactly the blocks a hidden size needs.
template <int KV>
__device__ __noinline__ void pro_norm_quant(const float* src, const __half* emb_row,
                                            const float* __restrict__ w, int n, float eps,
                                            StepShared& S, float* sq, uint4* q_s, int2* sb_s,
                                            const hv_step_desc& D, int mark) {
  const int n4 = n / 4;
  const int t = threadIdx.x;
  float4 xv[KV], wv[KV];
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int i4 = t + k * kConsThreads;
    if (i4 < n4) {
      if (src) {
        xv[k] = __ldcg(reinterpret_cast<const float4*>(src) + i4);
      } else {
        const __half2* e = reinterpret_cast<const __half2*>(emb_row) + 2 * i4;
        const float2 a = __half22float2(e[0]), b = __half22float2(e[1]);
        xv[k] = make_float4(a.x, a.y, b.x, b.y);
      }
      wv[k] = __ldg(reinterpret_cast<const float4*>(w) + i4);
    } else {
      xv[k] = wv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int i4 = t + k * kConsThreads;
    if (i4 < n4)
      reinterpret_cast<float4*>(sq)[i4] =
          make_float4(__fmul_rn(xv[k].x, xv[k].x), __fmul_rn(xv[k].y, xv[k].y),
                      __fmul_rn(xv[k].z, xv[k].z), __fmul_rn(xv[k].w, xv[k].w));
  }
  csync();
  if (mark >= 0) trace_mark(D, mark);
  const float ss = block_pw_sum<CSync>(sq, &S.P.pw_hid, S.leafval, S.red);
  if (mark >= 0) trace_mark(D, mark + 1);
  const float d = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps));
#pragma unroll
  for (int k = 0; k < KV; ++k)
    xv[k] = make_float4(
        __fmul_rn(wv[k].x, __fdiv_rn(xv[k].x, d)), __fmul_rn(wv[k].y, __fdiv_rn(xv[k].y, d)),
        __fmul_rn(wv[k].z, __fdiv_rn(xv[k].z, d)), __fmul_rn(wv[k].w, __fdiv_rn(xv[k].w, d)));
  unsigned* q32 = reinterpret_cast<unsigned*>(q_s);
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int i4 = t + k * kConsThreads;
    if (i4 < n4) {                      // uniform over each 8-lane group (n4 % 8 == 0)
      float sc;
      int bs;
      q32[i4] = quant_block_8lanes(xv[k], &sc, &bs);
      if ((i4 & 7) == 0) sb_s[i4 >> 3] = make_int2(__float_as_int(sc), bs);
    }
  }
  csync();
}

// The hidden-size dispatch of pro_norm_quant (n <= kMaxHidden).
HV_DEV void norm_quant(const float* src, const __half* emb_row, const float* w, int n,
                       float eps, StepShared& S, float* sq, uint4* q_s, int2* sb_s,
                       const hv_step_desc& D, int mark) {
  const int kv = (n / 4 + kConsThreads - 1) / kConsThreads;
  if (kv <= 2) pro_norm_quant<2>(src, emb_row, w, n, eps, S, sq, q_s, sb_s, D, mark);
  else if (kv <= 4) pro_norm_quant<4>(src, emb_row, w, n, eps, S, sq, q_s, sb_s, D, mark);
  else if (kv <= 5) pro_norm_quant<5>(src, emb_row, w, n, eps, S, sq, q_s, sb_s, D, mark);
  else pro_norm_quant<kMaxHidden / 4 / kConsThreads>(src, emb_row, w, n, eps, S, sq, q_s, sb_s, D, mark);
}

// act <- a vector other CTAs already quantised: int8 [n] at q, then (scale, sum) pairs
// for its n / 32 blocks at sb (read through L2).
__device__ __noinline__ void pro_load_quant(const void* q, const int2* sb, int n, uint4* q_s,
                                            int2* sb_s) {
  const uint4* q4 = reinterpret_cast<const uint4*>(q);
  for (int i = threadIdx.x; i < n / 16; i += kConsThreads) q_s[i] = __ldcg(q4 + i);
  for (int i = threadIdx.x; i < n / kBlock; i += kConsThreads) sb_s[i] = __ldcg(sb + i);
  csync();
}

// The CTA's SiLU outputs, staged in shared memory (nval values starting at element
// first, first % 32 == 0, nval % 32 == 0), quantised per 32 (8 lanes per block) into
// int8 q[first ..] and (scale, sum) sb[first / 32 ..] in global memory.
__device__ __noinline__ void quant_staged(const float* vals, int nval, int first, int8_t* q,
                                          int2* sb) {
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const int nb = nval / kBlock;
  for (int base = (threadIdx.x >> 5) * 4; base < nb; base += kConsWarps * 4) {
    const int b = base + (lane >> 3);
    if (b < nb) {                      // uniform over each 8-lane group
      const float4 v = reinterpret_cast<const float4*>(vals)[b * 8 + sub];
      const unsigned w = quant4(v, v, 1.0f, false, first / kBlock + b, sub == 0, sb);
      reinterpret_cast<unsigned*>(q + first)[b * 8 + sub] = w;
    }
  }
}


// Sharded head: every rank's winner (value, global index) goes into every rank's
// exchange row [rank]; once all `world` rows carry this launch's sequence number, the
// overall winner (lowest index on ties, as np.argmax) is the same on every rank. The
// sequence number is a launch counter kept in row HV_MAX_WORLD of the local exchange
// array (every rank makes the same launches, so the counters agree). One thread; the
// wait is bounded (false and HV_E_TIMEOUT when it runs out).
HV_DEV bool exchange_argmax(const hv_step_desc& D, int rank, int world, float* v, int* idx) {
  int32_t* mine = D.peers->xchg[rank];
  const int seq = mine[HV_MAX_WORLD * 4] + 1;
  mine[HV_MAX_WORLD * 4] = seq;
  for (int k = 0; k < world; ++k) {
    int32_t* row = D.peers->xchg[k] + rank * 4;
    row[0] = __float_as_int(*v);
    row[1] = *idx;
  }
  __threadfence_system();
  for (int k = 0; k < world; ++k)
    asm volatile("st.release.sys.global.s32 [%0], %1;" :: "l"(D.peers->xchg[k] + rank * 4 + 2),
                 "r"(seq) : "memory");
  const unsigned long long t0 = global_ns();
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int j = 0; j < world; ++j) {
    const unsigned* flag = reinterpret_cast<const unsigned*>(mine + j * 4 + 2);
    while ((int)ld_acquire_sys(flag) != seq) {
      if (global_ns() - t0 > kWaitNs) {
        atomicCAS(D.status, 0, HV_E_TIMEOUT);
        return false;
      }
    }
    const float cv = __int_as_float(__ldcv(mine + j * 4));
    const int ci = __ldcv(mine + j * 4 + 1);
    if (cv > bv || (cv == bv && ci < bi)) { bv = cv; bi = ci; }
  }
  *v = bv;
  *idx = bi;
  return true;
}

// Copies n quantised values starting at element `first` (first, n multiples of 32) of a
// quantised vector of `len` elements (int8 [len], then (scale, sum) per 32) from this
// rank's buffer `mine` into every other rank's copy. Cooperative over the consumers.
__device__ __noinline__ void share_bytes(void* const* peers, int rank, int world,
                                         const int8_t* mine, int first, int n, int len) {
  const uint4* q = reinterpret_cast<const uint4*>(mine + first);
  const int2* sb = reinterpret_cast<const int2*>(mine + len) + first / kBlock;
  for (int k = 0; k < world; ++k) {
    if (k == rank) continue;
    int8_t* dst = reinterpret_cast<int8_t*>(peers[k]);
    uint4* dq = reinterpret_cast<uint4*>(dst + first);
    int2* dsb = reinterpret_cast<int2*>(dst + len) + first / kBlock;
    for (int i = threadIdx.x; i < n / 16; i += kConsThreads) dq[i] = q[i];
    for (int i = threadIdx.x; i < n / kBlock; i += kConsThreads) dsb[i] = sb[i];
  }
}

// ---- GEMV phases from the ring ----------------------------------------------------------

enum { kStore = 0, kResidual = 1, kSiluPair = 2, kHead = 3 };

// Where a GEMV phase's rows go. Row r of the CTA's matrix is global row row0 + r; with a
// sharded step (world > 1) the residual rows are also stored into every other rank's h.
struct OutCtx {
  float* out;
  int row0;
  int world, rank;
  const hv_step_peers* peers;
};

HV_DEV int pp_row_of(int tile, int g, int rows, int pair_ffn, bool* ok) {
  if (pair_ffn > 0) {
    const int p = tile * 4 + (g & 3);
    *ok = p < pair_ffn;
    return (g < 4) ? p : pair_ffn + p;
  }
  const int row = tile * 8 + g;
  *ok = row < rows;
  return row;
}

template <int MODE>
HV_DEV void gemv_epilogue(float y, int row, bool ok, const OutCtx& O, float* best_v,
                          int* best_i) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (MODE == kSiluPair) {
    const float up = __shfl_down_sync(0xFFFFFFFFu, y, 16);
    if (g < 4 && t == 0 && ok) O.out[row] = silu_mul1(y, up);
  } else if (t == 0 && ok) {
    if (MODE == kStore) {
      O.out[row] = y;
    } else if (MODE == kResidual) {
      const int gr = O.row0 + row;
      const float v = __fadd_rn(__ldcg(O.out + gr), y);
      O.out[gr] = v;
      for (int k = 0; k < O.world; ++k)
        if (k != O.rank) O.peers->h[k][gr] = v;
    } else {
      O.out[row] = y;
      const int gr = O.row0 + row;                      // global vocab index
      if (y > *best_v || (y == *best_v && gr < *best_i)) { *best_v = y; *best_i = gr; }
    }
  }
}

// Explicit shared-memory loads from 32-bit shared addresses. The phase functions are out
// of line and receive generic pointers, through which the compiler would emit generic
// loads (about twice the cost in the GEMV loop); these keep the hot loops on ld.shared.
HV_DEV unsigned sh_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
HV_DEV uint4 lds_u4(unsigned a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
HV_DEV uint2 lds_u2(unsigned a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
HV_DEV float4 lds_f4(unsigned a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
HV_DEV float2 lds_f2(unsigned a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}
HV_DEV float lds_f1(unsigned a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
HV_DEV void sts_f1(unsigned a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" :: "r"(a), "f"(v) : "memory");
}
HV_DEV void sts_f4(unsigned a, float x, float y, float z, float w) {
  asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" :: "r"(a), "f"(x), "f"(y), "f"(z), "f"(w)
               : "memory");
}

// Block terms of iteration u of a ring slot for the lane's row g: blocks 2t (x) and
// 2t+1 (y) of logical iteration `it` (the combine of gemv_tile8 in gemv_mma.cuh).
// sl, act_w and sb are shared addresses of the slot, the int8 activation words and the
// (scale, sum) pairs.
HV_DEV float2 slot_terms_sh(unsigned sl, int u, unsigned act_w, unsigned sb, int it, int g,
                            int t, int lane, int nvalid) {
  MmaLoads L;
  const uint4 a = lds_u4(sl + u * kPpNibWords * 4 + 16 * lane);
  const uint4 b = lds_u4(sl + u * kPpNibWords * 4 + 512 + 16 * lane);
  L.w[0] = a.x; L.w[1] = a.y; L.w[2] = a.z; L.w[3] = a.w;
  L.w[4] = b.x; L.w[5] = b.y; L.w[6] = b.z; L.w[7] = b.w;
  L.s = lds_f2(sl + kSlotScaleOff + u * kPpScales * 4 + 8 * lane);
  const uint2 bw = (g < nvalid) ? lds_u2(act_w + ((it * 8 + g) * 4 + t) * 8) : make_uint2(0u, 0u);
  int e, o;
  mma_iter(L.w, bw, t, nvalid, e, o);
  const uint4 sbp = lds_u4(sb + (it * 8 + 2 * t) * 8);   // blocks 2t and 2t+1: (s, sum) x 2
  float ce = 0.f, co = 0.f;
  if (2 * t < nvalid)
    ce = __fmul_rn(__fmul_rn(L.s.x, __int_as_float((int)sbp.x)), i2f_exact(e - 8 * (int)sbp.y));
  if (2 * t + 1 < nvalid)
    co = __fmul_rn(__fmul_rn(L.s.y, __int_as_float((int)sbp.z)), i2f_exact(o - 8 * (int)sbp.w));
  return make_float2(ce, co);
}


// slot_terms_sh over a slot of dq words (hv_w4_prepack_dq): lane (g, t) finds all four
// words of its blocks 2t and 2t+1 at the addresses where the tile-interleaved slot keeps
// word t of blocks 0..3 and 4..7, and forms their exact int32 dots with dp4a (block_dot)
// instead of the tensor-pipe MMAs; the terms are the same values. act_q: the int8
// activations, 32 bytes per block.
HV_DEV float2 slot_terms_dq(unsigned sl, int u, unsigned act_q, unsigned sb, int it, int t,
                            int lane, int nvalid) {
  const uint4 e = lds_u4(sl + u * kPpNibWords * 4 + 16 * lane);
  const uint4 o = lds_u4(sl + u * kPpNibWords * 4 + 512 + 16 * lane);
  const float2 s = lds_f2(sl + kSlotScaleOff + u * kPpScales * 4 + 8 * lane);
  const int be = it * 8 + 2 * t;
  const uint4 sbp = lds_u4(sb + be * 8);              // blocks 2t and 2t+1: (s, sum) x 2
  float ce = 0.f, co = 0.f;
  if (2 * t < nvalid) {
    const int d = block_dot(e, lds_u4(act_q + be * 32), lds_u4(act_q + be * 32 + 16),
                            (int)sbp.y);
    ce = __fmul_rn(__fmul_rn(s.x, __int_as_float((int)sbp.x)), i2f_exact(d));
  }
  if (2 * t + 1 < nvalid) {
    const int d = block_dot(o, lds_u4(act_q + be * 32 + 32), lds_u4(act_q + be * 32 + 48),
                            (int)sbp.w);
    co = __fmul_rn(__fmul_rn(s.y, __int_as_float((int)sbp.z)), i2f_exact(d));
  }
  return make_float2(ce, co);
}

// The block terms of one slot iteration in either weight arrangement.
template <bool kDq>
HV_DEV float2 slot_terms(unsigned sl, int u, unsigned act_w, unsigned sb, int it, int g, int t,
                         int lane, int nvalid) {
  if constexpr (kDq) return slot_terms_dq(sl, u, act_w, sb, it, t, lane, nvalid);
  else return slot_terms_sh(sl, u, act_w, sb, it, g, t, lane, nvalid);
}

// The CTA's tiles [t0, t1) of one GEMV phase, their slots starting at sequence number q0.
// Work items are (tile, leaf of numpy's pairwise recursion), tile-major like the ring;
// item k goes to warp k % 8, so every warp has work even when the CTA has few tiles
// (leaves are independent chains). An item walks its leaf's eight strided accumulators
// (the lane's 2t, 2t+1) with no branch per iteration, folds them across the quad
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) and, in the last leaf, adds the n % 8 tail in order.
// Single-leaf rows finish in the item; otherwise leaf values meet in `leafbuf` and one
// warp per tile folds them with the recursion's '+' (fold_leaves). A slot shared by two
// items (a leaf boundary inside it) gets half the release count from each.
// MODE kStore/kResidual/kHead: 8-row tiles of `rows` rows. kSiluPair: tiles of 4 gate
// rows (quads 0-3) and their 4 up rows (quads 4-7) of a [gate | up] matrix with pair_ffn
// rows per half; SiLU(gate) * up is formed in the lane that holds the gate row and stored
// at out[p - 4 t0] for pair p (a shared-memory staging buffer). kDq: the slots hold the
// dq arrangement of the words (slot_terms_dq).
template <int MODE, bool kDq>
__device__ __noinline__ void gemv_ring(const Ring R, unsigned q0, const GvPlan& P,
                                       const ActView act, int t0, int t1, int rows,
                                       int pair_ffn, const OutCtx O, float* best_v,
                                       int* best_i, float* leafbuf, StepShared& S,
                                       int* status) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int warp = threadIdx.x >> 5;
  const int niter = pp_iters(P.nb);
  const int spt = slots_per_tile(niter);
  const int nleaf = P.nleaf, nfull = P.nfull, ntail = P.ntail;
  const int nitems = (t1 - t0) * nleaf;
  const unsigned act_w = sh_addr(act.q), sbs = sh_addr(act.sb);
  bool failed = false;
  for (int k = warp; k < nitems && !failed; k += kConsWarps) {
    const int lt = k / nleaf, lf = k - lt * nleaf;
    const int ia = lf == 0 ? 0 : P.it_end[lf - 1];
    const int ib = lf == nleaf - 1 ? niter : P.it_end[lf];   // the last leaf owns the tail
    const int ifull = min(ib, nfull);
    // numpy assigns a leaf's first term and adds the rest; starting from -0.0 and adding
    // every term gives the same bits ((-0) + x == x for every x, -0 and +0 included), so
    // the loop needs no peeled first iteration
    float ae = -0.0f, ao = -0.0f;
    float2 tail = make_float2(0.f, 0.f);
    for (int s0 = ia - ia % kSlotIters; s0 < ib; s0 += kSlotIters) {
      const int s1 = min(s0 + kSlotIters, niter);
      const unsigned q = q0 + slot_seq(lt, s0 / kSlotIters, t1 - t0, spt, nleaf == 1);
      if (!warp_wait(R.full_of(q), R.parity(q), S, status)) {
        failed = true;
        break;
      }
      const unsigned sl = sh_addr(R.slot(q));
      const int a = max(ia, s0), bb = min(ib, s1), bf = min(bb, ifull);
      if (a == s0 && bf == s0 + kSlotIters) {       // the whole slot: fixed trip count
#pragma unroll
        for (int u = 0; u < kSlotIters; ++u) {
          const float2 v = slot_terms<kDq>(sl, u, act_w, sbs, s0 + u, g, t, lane, 8);
          ae = __fadd_rn(ae, v.x);
          ao = __fadd_rn(ao, v.y);
        }
      } else {
        for (int it = a; it < bf; ++it) {
          const float2 v = slot_terms<kDq>(sl, it - s0, act_w, sbs, it, g, t, lane, 8);
          ae = __fadd_rn(ae, v.x);
          ao = __fadd_rn(ao, v.y);
        }
      }
      if (bb > bf) tail = slot_terms<kDq>(sl, bf - s0, act_w, sbs, bf, g, t, lane, ntail);
      __syncwarp();
      const bool shared = ia > s0 || ib < s1;
      if (lane == 0) mbar_arrive_n(R.empty_of(q), shared ? kConsWarps / 2 : kConsWarps);
    }
    if (failed) break;
    float v = (ifull > ia) ? quad_fold(ae, ao) : 0.f;
    if (lf == nleaf - 1) {
      for (int j = 0; j < ntail; ++j) {
        const float x =
            __shfl_sync(0xFFFFFFFFu, (j & 1) ? tail.y : tail.x, (lane & ~3) | (j >> 1));
        v = __fadd_rn(v, x);
      }
    }
    if (nleaf == 1) {
      bool ok;
      int row = pp_row_of(t0 + lt, g, rows, pair_ffn, &ok);
      if (MODE == kSiluPair) row -= 4 * t0;            // staged in shared memory
      gemv_epilogue<MODE>(__fadd_rn(0.0f, v), row, ok, O, best_v, best_i);
    } else if (t == 0) {
      leafbuf[((size_t)lt * 8 + g) * nleaf + lf] = v;
    }
  }
  if (nleaf > 1) {
    csync();
    for (int lt = warp; lt < t1 - t0 && !failed; lt += kConsWarps) {
      bool ok;
      int row = pp_row_of(t0 + lt, g, rows, pair_ffn, &ok);
      if (MODE == kSiluPair) row -= 4 * t0;
      const float y = fold_leaves(P, leafbuf + ((size_t)lt * 8 + g) * nleaf);
      gemv_epilogue<MODE>(y, row, ok, O, best_v, best_i);
    }
  }
}

// ---- attention: the reference's order, bit for bit (attn_exact.cuh) ---------------------
//
// Phase A, per (kv head, chunk) work item: q/k RMSNorm + RoPE of the item's heads, the KV
// append (by the chunk holding pos), then every position's dot with the GS query heads in
// OpenBLAS's row-dot order, K rows from the ring. Scores go to D.part [head][cap], the
// chunk's maximum per head to D.part [n_head][cap ..][chunk]; then the item adds one to
// its kv head's ticket.
// Phase B, per (kv head, 32-dim slice) on its own CTA, as soon as all nch chunks of the
// kv head have arrived (ticket; no grid barrier): the maximum, numpy's pairwise sum of
// the exps, then one warp per query head runs the sequential weighted V sum over V rows
// that the producer brings into the ring as 32-dim slices (tensor copies), row pos from
// this step's qkv; the warp quantises its 32 outputs (one quant_a8s block) into ctx.

// One cache element at shared address a, as a float (binary16 widens exactly).
template <class KT>
HV_DEV float slot_elem(unsigned a) {
  if constexpr (kKvHalf<KT>) {
    unsigned short h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a));
    return __half2float(__ushort_as_half(h));
  } else {
    return lds_f1(a);
  }
}

// Element e of a cache row held in shared memory (a ring slot row of KT, or a float row).
template <class KT>
struct SlotRow {
  unsigned addr;
  bool f32row;                                     // this step's row, kept as floats
  HV_DEV float operator()(int e) const {
    if constexpr (kKvHalf<KT>) {
      if (!f32row) {
        unsigned short h;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr + 2u * e));
        return __half2float(__ushort_as_half(h));
      }
    }
    return lds_f1(addr + 4u * e);
  }
};

// Phase A of this CTA's (kv head, chunk) item -- at most one per CTA (the host checks
// n_kv * attn_chunks <= grid), because an item waits for the other chunks of its kv head.
// Chunk c is node c of numpy's recursion over the T = pos + 1 positions cut at the
// launch's depth (S.front), so its pairwise sum is an exact subtree of the softmax sum.
// Steps: q/k norm + RoPE, the KV append (the last chunk holds pos), the scores (OpenBLAS's
// row-dot order, K rows from the ring), the chunk's maximum per head to global memory and
// one count on the kv head's first ticket; once every chunk of the kv head has counted,
// M = their maximum, e_t = np_expf(s_t - M) for the chunk's rows (to D.part's exp rows)
// and the chunk's pairwise sum per head (to D.part's node sums); one count on the second
// ticket.
template <int GS, class KT>
__device__ __noinline__ bool attn_scores_ring(const hv_step_desc& D, const hv_layer_w* L,
                                              int pos, int layer, const Ring R, unsigned* qp,
                                              StepShared& S, PwTree* tree, float* area,
                                              int tb) {
  const int nkv = D.n_kv, nch = D.attn_chunks, cap = D.cap, nq = D.n_head;
  const int wi = blockIdx.x;
  if (wi >= nkv * nch) return true;
  const StepScratch X = step_scratch(D);
  float* q_s = area;
  float* kpos_s = q_s + GS * kHd;
  float* vpos_s = kpos_s + kHd;
  float* tmp_s = vpos_s + kHd;                       // (GS + 1) x 128
  float* m_s = tmp_s + (GS + 1) * kHd;               // GS maxima (+ pad)
  float* lg_s = m_s + 8;                             // [chunk_max][GS]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7, rr = lane >> 3;
  const float* cs = D.cos_t + (size_t)pos * (kHd / 2);
  const float* sn = D.sin_t + (size_t)pos * (kHd / 2);
  const float scale = D.attn_scale;
  constexpr int HP = GS < 4 ? GS : 4;
  const int g = wi / nch, c = wi % nch;
  const int T = pos + 1;
  int t0, t1, te;
  front_rows(S.front, pos, c, &t0, &t1, &te);
  const int n = t1 - t0;
  const int nk = (te - t0 + kSlotRows - 1) / kSlotRows;
  const unsigned qk = *qp;
  *qp += (unsigned)nk;
  // GS query heads, the kv head's k (normed + rotated) and its raw v, a warp each
  for (int h = warp; h < GS + 2; h += kConsWarps) {
    if (h < GS) {
      warp_norm_rope(D.qkv + (size_t)(g * GS + h) * kHd, L->qn, cs, sn, D.eps,
                     tmp_s + h * kHd, q_s + h * kHd);
    } else if (h == GS) {
      warp_norm_rope(D.qkv + (size_t)(nq + g) * kHd, L->kn, cs, sn, D.eps,
                     tmp_s + GS * kHd, kpos_s);
      if constexpr (kKvHalf<KT>) {
        float4* k4 = reinterpret_cast<float4*>(kpos_s) + lane;
        *k4 = round_half4(*k4);
      }
    } else {
      float4 v4 =
          __ldcg(reinterpret_cast<const float4*>(D.qkv + (size_t)(nq + nkv + g) * kHd) + lane);
      if constexpr (kKvHalf<KT>) v4 = round_half4(v4);
      reinterpret_cast<float4*>(vpos_s)[lane] = v4;
    }
  }
  if (layer == 0 && warp == kConsWarps - 1) {        // this chunk's subtree, for the launch
    const bool built = n == 0 || pw_tree_build_warp(n, tree);
    if (lane == 0) S.tree_ok = built;
  }
  csync();
  trace_mark(D, tb + 14);
  trace_wait(D, S, tb + 20);
  if (n > 0 && t1 == T && threadIdx.x < kHd) {       // the chunk holding pos appends
    KT* kc = reinterpret_cast<KT*>(L->kc) + (size_t)g * cap * kHd;
    KT* vc = reinterpret_cast<KT*>(L->vc) + (size_t)g * cap * kHd;
    kc[(size_t)pos * kHd + threadIdx.x] = to_kv<KT>(kpos_s[threadIdx.x]);
    vc[(size_t)pos * kHd + threadIdx.x] = to_kv<KT>(vpos_s[threadIdx.x]);
  }

  // scores: block m = positions [t0 + 20 m, +20) (one ring slot of K rows; row pos from
  // kpos_s) to warp m % 8, four positions per pass (8 lanes each)
  bool ok = true;
  const int nblk = (n + kSlotRows - 1) / kSlotRows;
  float qr[HP][16];
  if constexpr (GS <= 4) load_qregs<HP>(q_s, j, qr);
  for (int m = warp; m < nblk && ok; m += kConsWarps) {
    const int r0 = t0 + m * kSlotRows, r1 = min(r0 + kSlotRows, t1);
    unsigned slot = 0;
    if (m < nk) {
      const unsigned q = qk + (unsigned)m;
      ok = warp_wait(R.full_of(q), R.parity(q), S, D.status);
      if (!ok) break;
      slot = sh_addr(R.slot(q));
    }
    const long long c0 = clock64();
    const RunWin rw = run_window(S.runs, r0);
#pragma unroll 1
    for (int p0 = 0; p0 < GS; p0 += HP) {
      if constexpr (GS > 4) load_qregs<HP>(q_s + p0 * kHd, j, qr);
#pragma unroll 1
      for (int tg = r0; tg < r1; tg += 4) {
        const int t = tg + rr;
        const bool valid = t < r1;
        const bool cached = t < te;
        const int kind = valid ? kind_in(rw, t) : 0;
        SlotRow<KT> row;
        row.f32row = !cached;
        row.addr = cached ? slot + (unsigned)((t - r0) * kHd * (int)sizeof(KT)) : sh_addr(kpos_s);
        float d[HP];
        rowdots_blas<HP>(row, kind, qr, q_s + p0 * kHd, j, d);
        float v = d[0];
#pragma unroll
        for (int h = 1; h < HP; ++h) v = (j == h) ? d[h] : v;
        if (valid && j < HP) lg_s[(t - t0) * GS + p0 + j] = __fmul_rn(v, scale);
      }
    }
    if (lane == 0) S.busy[warp] += clock64() - c0;
    if (m < nk) {
      __syncwarp();
      if (lane == 0) mbar_arrive_n(R.empty_of(qk + (unsigned)m), kConsWarps);
    }
  }
  csync();
  trace_mark(D, tb + 15);
  trace_wait(D, S, tb + 21);
  if (threadIdx.x == 0 && D.trace != nullptr) {
    D.trace[(size_t)blockIdx.x * HV_STEP_TRACE_STRIDE(D.n_layer) + tb + 25] = S.busy[0];
    S.busy[0] = 0;
  }
  if (!S.tree_ok) {
    if (threadIdx.x == 0) {
      atomicCAS(D.status, 0, HV_E_INVALID);
      *(volatile int*)&S.abort = 1;
    }
    return false;
  }
  // the chunk's maximum per head, then the first ticket
  for (int i = warp; i < GS; i += kConsWarps) {
    float mx = -INFINITY;
    for (int t = lane; t < n; t += 32) mx = fmaxf(mx, lg_s[t * GS + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) X.cmax[(size_t)(g * GS + i) * nch + c] = mx;
  }
  csync();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(D.ticket + g, 1);
    S.ok = wait_count(D.ticket + g, (unsigned)((layer + 1) * nch), D.status);
    if (!S.ok) *(volatile int*)&S.abort = 1;
  }
  csync();
  if (!S.ok) return false;
  trace_mark(D, tb + 16);
  // M per head over every chunk of the kv head; the exps in place and to global memory
  for (int i = warp; i < GS; i += kConsWarps) {
    float mx = -INFINITY;
    for (int k = lane; k < nch; k += 32) mx = fmaxf(mx, __ldcg(X.cmax + (size_t)(g * GS + i) * nch + k));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) m_s[i] = mx;
  }
  csync();
  for (int i = 0; i < GS; ++i) {
    const float M = m_s[i];
    float* eg = X.exps + (size_t)(g * GS + i) * X.ew + t0;
    for (int t = threadIdx.x; t < n; t += kConsThreads) {
      const float e = np_expf(__fsub_rn(lg_s[t * GS + i], M));
      lg_s[t * GS + i] = e;
      eg[t] = e;
    }
  }
  csync();
  // the chunk's pairwise sum per head: leaves by 8-lane groups, then one warp per head
  if (n > 0) {
    const int ngr = kConsWarps * 4, gi = warp * 4 + (lane >> 3);
    const int nvl = (pw_tree_nodes_max(front_chunk_max(cap, nch)) + 3) & ~3;
    float* vals = lg_s + (((size_t)n * GS + 3) & ~size_t(3));   // [GS][nvl]
    for (int pl = gi; pl < ((tree->nleaf * GS + ngr - 1) / ngr) * ngr; pl += ngr) {
      const bool live = pl < tree->nleaf * GS;
      const int i = live ? pl % GS : 0, l = live ? pl / GS : 0;
      const int id = tree->leaf[l];
      const float v = leaf_sum_strided(lg_s + i, GS, live ? (int)tree->start[id] : 0,
                                       live ? (int)tree->size[id] : 1, lane & 7);
      if (live && (lane & 7) == 0) vals[(size_t)i * nvl + id] = v;
    }
    csync();
    for (int i = warp; i < GS; i += kConsWarps) {
      const float sum = pw_tree_fold_raw(tree, vals + (size_t)i * nvl);
      if (lane == 0) X.nsum[(size_t)(g * GS + i) * nch + c] = sum;
    }
  }
  csync();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(D.ticket + nkv + g, 1);
  }
  trace_mark(D, tb + 17);
  return true;
}

// Phase B of this CTA's items (query head h, 32-dim slice): once every chunk of h's kv
// head has its exps and subtree sums in (the second ticket), S = the top of the
// recursion over the chunks' sums; then the sequential weighted V sum
// acc_d = (((+0 + w_0 v_0[d]) + w_1 v_1[d]) + ...), w_t = e_t / S, one chain of T adds per
// output element. Block k's ring slot holds V rows [64 k, 64 k + 64) of the slice and h's
// exps for the same rows. Block u (counted over the launch) goes to helper u % 4: it
// divides the block's exps by S, forms the products (row pos's v from this step's qkv,
// +0 past it: the chain never holds -0, so +0 terms leave it unchanged) and stores them
// transposed into its own products buffer, dim-major, four rows per 16 bytes. Warp 0
// (the chain) loads each half of block k + 1 as soon as the adds of the same half of
// block k are issued: 16 loads and 64 dependent adds per block, nothing else on its
// sub-partition.
template <int GS, class KT>
__device__ __noinline__ bool attn_ctx_ring(const hv_step_desc& D, int pos, int layer,
                                           const Ring R, unsigned* qp, StepShared& S,
                                           float* area, int tb) {
  const int nkv = D.n_kv, nch = D.attn_chunks, nq = D.n_head;
  const int nitems = nq * kSlices;
  constexpr int BR = kCtxRows;
  constexpr int kVB = BR * 32 * (int)sizeof(KT);     // bytes of the V part of a slot
  constexpr int kRowB = 32 * (int)sizeof(KT);        // bytes of one 32-dim row slice
  constexpr unsigned kPB = kCtxPFloats * 4;          // bytes of one products buffer
  const StepScratch X = step_scratch(D);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hw = ctx_helper(warp);
  const int T = pos + 1;
  const int nblk = (T + BR - 1) / BR;
  const int nch4 = (nch + 3) & ~3;
  float* vals = area;                                // [nch] the chunks' sums
  float* s_s = vals + nch4;                          // S
  float* pbuf = s_s + 4;                             // [kCtxPBufs][32][kCtxPStride]
  float* wsc = pbuf + kCtxPBufs * kCtxPFloats;       // [kCtxHelpers][64] weights
  if (ctx_item(blockIdx.x, gridDim.x, nitems, 0) < 0) return true;
  bool ok = true;
  for (int j = 0;; ++j) {
    const int item = ctx_item(blockIdx.x, gridDim.x, nitems, j);
    if (item < 0) break;
    const int h = item / kSlices, jsl = item % kSlices, g = h / GS;
    const unsigned qv0 = *qp;
    *qp += (unsigned)nblk;
    if (threadIdx.x == 0) {
      S.ok = wait_count(D.ticket + nkv + g, (unsigned)((layer + 1) * nch), D.status);
      if (!S.ok) *(volatile int*)&S.abort = 1;
    }
    csync();
    if (!S.ok) return false;
    if (j == 0) trace_mark(D, tb + 18);
    const unsigned u0 = S.pseq;                      // blocks of earlier items this launch
    const int nf = S.front.n;
    for (int e = threadIdx.x; e < nf; e += kConsThreads)
      vals[e] = __ldcg(X.nsum + (size_t)h * nch + e);
    csync();
    if (threadIdx.x == 0) {
      s_s[0] = pw_front_fold(S.front, vals);
      S.pseq = u0 + (unsigned)nblk;
    }
    csync();
    const float S_ = s_s[0];
    const unsigned pb = sh_addr(pbuf);
    if (warp == 0) {
      // the chain: lane = dim 32 jsl + lane of head h
      float acc = 0.0f;
      const unsigned pl = pb + (unsigned)(lane * kCtxPStride * 4);
      if (lane == 0) S.wait[0] = 0;
      // rows 0-31 (r0) and 32-63 (r1) of the block being added; the next block's halves
      // are loaded into each as soon as its adds are issued
      constexpr int H = BR / 8;                      // float4 per half block
      float4 r0[H], r1[H];
      auto wait_blk = [&](int k) -> unsigned {      // shared address of block k's products
        const unsigned u = u0 + (unsigned)k, b = u % kCtxPBufs;
        ok = warp_wait(S.pfull + b, (u / kCtxPBufs) & 1u, S, D.status);
        return pl + b * kPB;
      };
      auto load = [&](unsigned a, float4* r) {
#pragma unroll
        for (int x = 0; x < H; ++x) r[x] = lds_f4(a + 16u * (unsigned)x);
      };
      auto adds = [&](const float4* r) {
#pragma unroll
        for (int x = 0; x < H; ++x) {
          acc = __fadd_rn(acc, r[x].x);
          acc = __fadd_rn(acc, r[x].y);
          acc = __fadd_rn(acc, r[x].z);
          acc = __fadd_rn(acc, r[x].w);
        }
      };
      const unsigned a0 = wait_blk(0);
      if (ok) {
        load(a0, r0);
        load(a0 + 16u * H, r1);
      }
#pragma unroll 1
      for (int k = 0; k < nblk && ok; ++k) {
        adds(r0);
        const bool more = k + 1 < nblk;
        unsigned an = 0;
        if (more) {
          an = wait_blk(k + 1);
          if (!ok) break;
          load(an, r0);
        }
        adds(r1);
        if (more) load(an + 16u * H, r1);
        // block k's loads completed long ago: its buffer goes back to its helper
        __syncwarp();
        if (lane == 0) mbar_arrive_n(S.pfree + (u0 + (unsigned)k) % kCtxPBufs, 1);
      }
      if (lane == 0) S.ctx_wait_ns += S.wait[0];
      if (ok) {
        // ctx element (head h, dim 32 jsl + lane) -> int8 + (scale, sum) of its block
        const int world = D.world > 1 ? D.world : 1, rank = world > 1 ? D.rank : 0;
        const int qall = nq * kHd * world;
        const int idx = (rank * nq + h) * kHd + 32 * jsl + lane;
        int8_t q8;
        float sc;
        int bs;
        quant_block_warp(acc, lane, &q8, &sc, &bs);
        const int2 sbv = make_int2(__float_as_int(sc), bs);
        for (int k = 0; k < world; ++k) {
          int8_t* cq = reinterpret_cast<int8_t*>(world > 1 ? D.peers->ctx[k] : (void*)D.ctx);
          cq[idx] = q8;
          if (lane == 0) reinterpret_cast<int2*>(cq + qall)[idx / kBlock] = sbv;
        }
      }
    } else if (hw >= 0) {
      // a helper: every fourth block, all 64 rows; lane = dim
      float vpos = __ldcg(D.qkv + (size_t)(nq + nkv + g) * kHd + 32 * jsl + lane);
      if constexpr (kKvHalf<KT>) vpos = __half2float(__float2half_rn(vpos));
      const unsigned wl = sh_addr(wsc + hw * BR);
      const unsigned pl = pb + (unsigned)(hw * kCtxPFloats + lane * kCtxPStride) * 4u;
      if (lane == 0) S.wait[warp] = 0;
      const int kfirst = (int)(((unsigned)hw + kCtxHelpers - u0 % kCtxHelpers) % kCtxHelpers);
#pragma unroll 1
      for (int k = kfirst; k < nblk && ok; k += kCtxHelpers) {
        const unsigned q = qv0 + (unsigned)k;
        const unsigned c = (u0 + (unsigned)k) / kCtxPBufs;   // this buffer's use number
        ok = warp_wait(R.full_of(q), R.parity(q), S, D.status);
        if (!ok) break;
        const unsigned sl = sh_addr(R.slot(q));
        const int t0 = k * BR;                       // position of the block's first row
        {
          const float e0 = lds_f1(sl + (unsigned)(kVB + 4 * lane));
          const float e1 = lds_f1(sl + (unsigned)(kVB + 4 * (32 + lane)));
          sts_f1(wl + 4u * (unsigned)lane, t0 + lane < T ? __fdiv_rn(e0, S_) : 0.0f);
          sts_f1(wl + 4u * (unsigned)(32 + lane), t0 + 32 + lane < T ? __fdiv_rn(e1, S_) : 0.0f);
        }
        __syncwarp();
        float p[BR];
        const unsigned vl = sl + (unsigned)(lane * (int)sizeof(KT));
#pragma unroll
        for (int x = 0; x < BR; ++x) p[x] = slot_elem<KT>(vl + (unsigned)(x * kRowB));
        const bool tail = t0 + BR > pos;             // the block holds row pos (or rows past it)
#pragma unroll
        for (int x = 0; x < BR; x += 4) {
          const float4 w4 = lds_f4(wl + 4u * (unsigned)x);
          const float w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            const int t = t0 + x + y;
            p[x + y] = !tail || t < pos ? __fmul_rn(w[y], p[x + y])
                     : t == pos          ? __fmul_rn(w[y], vpos)
                                         : 0.0f;
          }
        }
        // the slot is read (the products depend on every load): release it
        __syncwarp();
        if (lane == 0) mbar_arrive_n(R.empty_of(q), (unsigned)kConsWarps);
        if (c > 0) {
          ok = warp_wait(S.pfree + hw, (c - 1) & 1u, S, D.status);
          if (!ok) break;
        }
#pragma unroll
        for (int x = 0; x < BR; x += 4) sts_f4(pl + 4u * (unsigned)x, p[x], p[x + 1], p[x + 2], p[x + 3]);
        __syncwarp();
        if (lane == 0) mbar_arrive_n(S.pfull + hw, 1);
      }
      if (hw == 0 && lane == 0) S.ctx_sum_ns += S.wait[warp];
    }
    csync();
    if (!ok || *(volatile int*)&S.abort) return false;
  }
  trace_mark(D, tb + 19);
  return *(volatile int*)&S.abort == 0;
}

// ---- the kernel ------------------------------------------------------------------------

template <int GS, class KT, bool kDq>
__global__ void __launch_bounds__(kStepThreads, 1)
k_step(const hv_step_desc D, int flags, int nslots, int inflight, int evict_first, int runs,
       const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(128) unsigned char smem[];
  // sharded: n_head, n_kv, ffn and head_rows are this rank's; hidden, the o projection's
  // input (qdim) and the down projection's input (ffn_all) are whole
  const int world = D.world > 1 ? D.world : 1, rank = world > 1 ? D.rank : 0;
  const int hid = D.hidden, ffn = D.ffn, qdim = D.n_head * kHd * world, ffn_all = ffn * world;
  const int hrows = hid / world;
  const StepLayout Lo =
      step_layout(GS, hid, qdim, ffn_all, D.cap, D.attn_chunks, nslots, D.n_layer);
  StepShared& S = *reinterpret_cast<StepShared*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lo.bars);
  uint4* q_s = reinterpret_cast<uint4*>(smem + Lo.act_q);
  int2* sb_s = reinterpret_cast<int2*>(smem + Lo.act_sb);
  float* work = reinterpret_cast<float*>(smem + Lo.work);
  const Ring R{smem + Lo.ring, bars, bars + kMaxSlots, nslots};
  hv_layer_w* Ls = reinterpret_cast<hv_layer_w*>(smem + Lo.layers);
  PwTree* tree = reinterpret_cast<PwTree*>(smem + Lo.tree);
  const ActView act{q_s, sb_s};

  trace_mark(D, 0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < nslots; ++i) {
      mbar_init(R.full + i, 1);
      mbar_init(R.empty + i, kConsWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    S.abort = 0;
    // no barrier of this launch can complete before this CTA arrives, so the counter's
    // top bit is still the one the previous launch left
    S.phase = ld_acquire(D.barrier) & 0x80000000u;
    // sharded: neither word can move before this CTA has arrived (the cross-rank counter
    // flips only when this rank's CTA 0 arrives, which waits for this CTA)
    S.xphase = D.world > 1 ? ld_acquire_sys(D.barrier + 1) & 0x80000000u : 0u;
    S.gen = D.world > 1 ? ld_acquire(D.barrier + 2) : 0u;
    for (int w = 0; w < kConsWarps; ++w) S.wait[w] = 0, S.busy[w] = 0;
    S.ctx_wait_ns = 0;
    S.ctx_sum_ns = 0;
    for (int b = 0; b < kCtxPBufs; ++b) {
      mbar_init(S.pfull + b, 1);
      mbar_init(S.pfree + b, 1);
    }
    S.pseq = 0;
  }
  {
    const int* src = reinterpret_cast<const int*>(D.plans);
    int* dst = reinterpret_cast<int*>(&S.P);
    for (int i = threadIdx.x; i < (int)(sizeof(StepPlans) / 4); i += blockDim.x) dst[i] = __ldg(src + i);
    // the layer table, so no phase starts with a pointer load from global memory
    const unsigned long long* ls = reinterpret_cast<const unsigned long long*>(D.layers);
    unsigned long long* ld = reinterpret_cast<unsigned long long*>(Ls);
    const int nw = D.n_layer * (int)(sizeof(hv_layer_w) / 8);
    for (int i = threadIdx.x; i < nw; i += blockDim.x) ld[i] = __ldg(ls + i);
  }
  const int pos = *D.pos;
  const int tok = *D.tok;
  if (threadIdx.x == 0) {
    // the attention chunks: numpy's recursion over pos + 1 positions cut at depth
    // log2(attn_chunks) (every CTA builds the same list)
    const int depth = 31 - __clz(D.attn_chunks);
    S.tree_ok = pos >= 0 && pos < D.cap && pw_front_build(pos + 1, depth, &S.front);
  }
  __syncthreads();
  if (pos < 0 || pos >= D.cap || tok < 0 || tok >= D.vocab || !S.tree_ok) {
    // every CTA reads the same values, so all leave here, before any copy or barrier
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(D.status, HV_E_INVALID);
    return;
  }
  if (threadIdx.x >= kConsThreads) {               // the producer warp: one lane copies
    if (threadIdx.x == kConsThreads)
      produce<GS, KT>(D, Ls, flags, pos, R, S, inflight, evict_first, &vmap);
    return;
  }

  // ---- consumers
  if (threadIdx.x == 0) blas_runs(pos + 1, runs, &S.runs);   // read after the first csync
  const int nqkv = (D.n_head + 2 * D.n_kv) * kHd;
  const __half* emb_row = reinterpret_cast<const __half*>(D.emb16) + (size_t)tok * hid;
  {
    const int r0 = (int)(((long long)blockIdx.x * hid) / gridDim.x);
    const int r1 = (int)(((long long)(blockIdx.x + 1) * hid) / gridDim.x);
    for (int i = r0 + threadIdx.x; i < r1; i += kConsThreads) D.h[i] = __half2float(emb_row[i]);
  }
  const int it_hid = pp_iters(hid / kBlock), it_q = pp_iters(qdim / kBlock),
            it_ffn = pp_iters(ffn_all / kBlock);
  const OutCtx o_qkv{D.qkv, 0, 1, 0, nullptr};
  const OutCtx o_h{D.h, rank * hrows, world, rank, D.peers};
  const OutCtx o_head{D.logits, rank * D.head_rows, 1, 0, nullptr};
  int8_t* const cq = reinterpret_cast<int8_t*>(D.ctx);     // int8 [qdim], then (s, sum)
  int8_t* const aq = reinterpret_cast<int8_t*>(D.act);     // int8 [ffn_all], then (s, sum)
  unsigned q = 0;
  int off = 0, t0, t1;
  if (threadIdx.x == 0) prefetch_vectors(Ls, hid, true);
  trace_mark(D, 1);
  for (int l = 0; l < D.n_layer; ++l) {
    const hv_layer_w* L = Ls + l;
    const int tb = 2 + 28 * l;
    // P1: qkv
    norm_quant(l == 0 ? nullptr : D.h, emb_row, L->an, hid, D.eps, S, work, q_s, sb_s, D,
                   tb + 26);
    trace_mark(D, tb + 0);
    trace_wait(D, S, tb + 20);
    phase_tiles(pp_tiles(nqkv, 0), &off, &t0, &t1);
    gemv_ring<kStore, kDq>(R, q, S.P.gv_hid, act, t0, t1, nqkv, 0, o_qkv, nullptr, nullptr, work,
                      S, D.status);
    q += (unsigned)((t1 - t0) * slots_per_tile(it_hid));
    trace_mark(D, tb + 1);
    trace_wait(D, S, tb + 23);
    if (!grid_sync(D, S, (flags & kFlagLocalQkvBarrier) == 0)) return;
    trace_mark(D, tb + 2);
    // P2: attention -- scores per (kv head, chunk), then the context per (kv head, slice)
    if (!attn_scores_ring<GS, KT>(D, L, pos, l, R, &q, S, tree, work, tb)) return;
    if (!attn_ctx_ring<GS, KT>(D, pos, l, R, &q, S, work, tb)) return;
    trace_mark(D, tb + 3);
    if (!grid_sync(D, S)) return;
    trace_mark(D, tb + 4);
    if (threadIdx.x == 0) prefetch_vectors(L, hid, false);
    // P3: o projection + residual
    pro_load_quant(cq, reinterpret_cast<const int2*>(cq + qdim), qdim, q_s, sb_s);
    trace_mark(D, tb + 5);
    phase_tiles(pp_tiles(hrows, 0), &off, &t0, &t1);
    gemv_ring<kResidual, kDq>(R, q, S.P.gv_o, act, t0, t1, hrows, 0, o_h, nullptr, nullptr, work,
                         S, D.status);
    q += (unsigned)((t1 - t0) * slots_per_tile(it_q));
    trace_mark(D, tb + 6);
    if (!grid_sync(D, S)) return;
    trace_mark(D, tb + 7);
    // P4: gate/up + SiLU
    norm_quant(D.h, nullptr, L->fn, hid, D.eps, S, work, q_s, sb_s, D, -1);
    trace_mark(D, tb + 8);
    trace_wait(D, S, tb + 20);
    gu_tiles(ffn, &off, &t0, &t1);
    {
      // SiLU outputs staged after the leaf values, then quantised by the CTA that made them
      const int nl = S.P.gv_hid.nleaf;
      float* act_s = work + (nl > 1 ? (size_t)(t1 - t0) * 8 * nl : 0);
      const OutCtx o_act{act_s, 0, 1, 0, nullptr};
      gemv_ring<kSiluPair, kDq>(R, q, S.P.gv_hid, act, t0, t1, 2 * ffn, ffn, o_act, nullptr,
                           nullptr, work, S, D.status);
      csync();
      const int first = rank * ffn + t0 * 4;               // this CTA's outputs, whole blocks
      quant_staged(act_s, (t1 - t0) * 4, first, aq, reinterpret_cast<int2*>(aq + ffn_all));
      if (world > 1) {
        csync();
        share_bytes(D.peers->act, rank, world, aq, first, (t1 - t0) * 4, ffn_all);
      }
    }
    q += (unsigned)((t1 - t0) * slots_per_tile(it_hid));
    trace_mark(D, tb + 9);
    trace_wait(D, S, tb + 24);
    if (!grid_sync(D, S)) return;
    trace_mark(D, tb + 10);
    if (threadIdx.x == 0) {
      if (l + 1 < D.n_layer) prefetch_vectors(L + 1, hid, true);
      else prefetch_l2(D.onorm, (size_t)hid * 4);
    }
    // P5: down + residual
    pro_load_quant(aq, reinterpret_cast<const int2*>(aq + ffn_all), ffn_all, q_s, sb_s);
    trace_mark(D, tb + 11);
    trace_wait(D, S, tb + 20);
    phase_tiles(pp_tiles(hrows, 0), &off, &t0, &t1);
    gemv_ring<kResidual, kDq>(R, q, S.P.gv_ffn, act, t0, t1, hrows, 0, o_h, nullptr, nullptr, work,
                         S, D.status);
    q += (unsigned)((t1 - t0) * slots_per_tile(it_ffn));
    trace_mark(D, tb + 12);
    trace_wait(D, S, tb + 20);
    if (!grid_sync(D, S)) return;
    trace_mark(D, tb + 13);
  }

  // every CTA has passed its last attention phase: the kv heads' tickets restart at zero
  if (blockIdx.x == 0 && threadIdx.x < 2 * D.n_kv) D.ticket[threadIdx.x] = 0;
  if (!(flags & HV_STEP_HEAD)) return;
  const int th = 2 + 28 * D.n_layer;
  norm_quant(D.h, nullptr, D.onorm, hid, D.eps, S, work, q_s, sb_s, D, -1);
  trace_mark(D, th + 0);
  phase_tiles(pp_tiles(D.head_rows, 0), &off, &t0, &t1);
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  gemv_ring<kHead, kDq>(R, q, S.P.gv_hid, act, t0, t1, D.head_rows, 0, o_head, &bv, &bi, work,
                   S, D.status);
  trace_mark(D, th + 1);
  if (!(flags & HV_STEP_ARGMAX)) return;

  // per-CTA argmax, then the last CTA to finish picks the token
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { S.sv[warp] = bv; S.si[warp] = bi; }
    csync();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kConsWarps; ++w)
        if (S.sv[w] > S.sv[0] || (S.sv[w] == S.sv[0] && S.si[w] < S.si[0])) {
          S.sv[0] = S.sv[w];
          S.si[0] = S.si[w];
        }
      D.amax_v[blockIdx.x] = S.sv[0];
      D.amax_i[blockIdx.x] = S.si[0];
      __threadfence();
      S.flag = (atomicAdd(D.ticket + 2 * D.n_kv, 1) == (int)gridDim.x - 1);
    }
    csync();
    if (S.flag && threadIdx.x == 0) {
      __threadfence();
      float v = -INFINITY;
      int idx = 0x7FFFFFFF;
      for (int c = 0; c < (int)gridDim.x; ++c) {
        const float cv = __ldcg(D.amax_v + c);
        const int ci = __ldcg(D.amax_i + c);
        if (cv > v || (cv == v && ci < idx)) { v = cv; idx = ci; }
      }
      if (world > 1 && !exchange_argmax(D, rank, world, &v, &idx)) return;
      *D.tok = idx;
      const int s = *D.step;
      if (s >= 0 && s <= D.cap) D.gen[s] = idx;      // gen holds cap + 1 entries
      *D.step = s + 1;
      *D.pos = pos + 1;
      D.ticket[2 * D.n_kv] = 0;
    }
  }
  trace_mark(D, th + 2);
}

// The step kernel for group size gs: variant 0 = f32 cache, 2 = binary16 cache, 3 = f32
// cache over dq weight tiles, 4 = binary16 cache over dq weight tiles.
template <class KT, bool kDq>
static void* step_fn_gs(int gs) {
  switch (gs) {
    case 1: return (void*)k_step<1, KT, kDq>;
    case 2: return (void*)k_step<2, KT, kDq>;
    case 4: return (void*)k_step<4, KT, kDq>;
    default: return (void*)k_step<8, KT, kDq>;
  }
}
static void* step_fn(int gs, int variant) {
  switch (variant) {
    case 2: return step_fn_gs<__half, false>(gs);
    case 3: return step_fn_gs<float, true>(gs);
    case 4: return step_fn_gs<__half, true>(gs);
    default: return step_fn_gs<float, false>(gs);
  }
}

// The V-slice tensor map of a cache view (rows of 128 elements of `esz` bytes), encoded
// once per (base, rows, element size) through the driver's cuTensorMapEncodeTiled.
typedef CUresult (*TmapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int vslice_map(const void* base, long long rows, int esz, int box_rows,
                      CUtensorMap* out) {
  static std::mutex mu;
  static TmapEncodeFn enc = nullptr;
  static const void* last_base = nullptr;
  static long long last_rows = 0;
  static int last_esz = 0, last_box = 0;
  static CUtensorMap last;
  std::lock_guard<std::mutex> lk(mu);
  if (base == last_base && rows == last_rows && esz == last_esz && box_rows == last_box) {
    *out = last;
    return HV_OK;
  }
  if (!enc) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    HV_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr));
    HV_REQUIRE(fn != nullptr && qr == cudaDriverEntryPointSuccess, HV_E_UNSUPPORTED,
               "hv_step_launch: the driver has no cuTensorMapEncodeTiled");
    enc = (TmapEncodeFn)fn;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)kHd, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kHd * (cuuint64_t)esz};
  const cuuint32_t box[2] = {32u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  const CUresult r = enc(&m, esz == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                         2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HV_REQUIRE(r == CUDA_SUCCESS, HV_E_INVALID,
             "hv_step_launch: cuTensorMapEncodeTiled failed (%d) for the KV view %p x %lld rows",
             (int)r, base, rows);
  last = m;
  last_base = base;
  last_rows = rows;
  last_esz = esz;
  last_box = box_rows;
  *out = m;
  return HV_OK;
}

// Ring slots that fit next to the fixed regions (0 if the fixed regions alone do not).
static int step_slots(int gs, int hid, int qdim, int ffn, int cap, int nch, int n_layer) {
  const StepLayout L = step_layout(gs, hid, qdim, ffn, cap, nch, 0, n_layer);
  if (L.ring >= (size_t)kSmemLimit) return 0;
  const int n = (int)(((size_t)kSmemLimit - L.ring) / kSlotBytes);
  return n > kMaxSlots ? kMaxSlots : n;
}

}  // namespace hv

using namespace hv;

extern "C" {

int hv_step_config(int n_kv, int group, int cap, int* grid, int* threads, size_t* smem,
                   int* chunks, size_t* part_floats) {
  HV_REQUIRE(n_kv > 0 && cap > 0 && grid && threads && chunks && part_floats, HV_E_INVALID,
             "hv_step_config: bad arguments");
  HV_REQUIRE(group == 1 || group == 2 || group == 4 || group == 8, HV_E_UNSUPPORTED,
             "hv_step_config: group size %d (1, 2, 4 or 8)", group);
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  *grid = sms;
  *threads = kStepThreads;
  HV_REQUIRE(cap <= kExactMaxCap, HV_E_UNSUPPORTED,
             "hv_step_config: cache of %d positions (at most %d)", cap, kExactMaxCap);
  const int nch = 1 << front_depth(n_kv, sms);
  *chunks = nch;
  *part_floats = step_part_floats(n_kv * group, cap, nch);
  if (smem) *smem = 0;
  return HV_OK;
}

int hv_step_plans(int hidden, int qdim, int ffn, void* host_buf, size_t len) {
  HV_REQUIRE(host_buf && len >= sizeof(StepPlans), HV_E_INVALID,
             "hv_step_plans: buffer of %zu bytes needed", sizeof(StepPlans));
  HV_REQUIRE(hidden > 0 && qdim > 0 && ffn > 0 && hidden % kBlock == 0 && qdim % kBlock == 0 &&
                 ffn % kBlock == 0, HV_E_INVALID, "hv_step_plans: bad geometry");
  StepPlans* P = static_cast<StepPlans*>(host_buf);
  memset(P, 0, sizeof(StepPlans));
  const bool ok = pw_make_plan(hidden, &P->pw_hid) && gv_make_plan(hidden / kBlock, &P->gv_hid) &&
                  gv_make_plan(qdim / kBlock, &P->gv_o) && gv_make_plan(ffn / kBlock, &P->gv_ffn);
  HV_REQUIRE(ok, HV_E_UNSUPPORTED, "hv_step_plans: reduction plan does not fit");
  return HV_OK;
}

int hv_step_plans_bytes(size_t* bytes) {
  HV_REQUIRE(bytes, HV_E_INVALID, "hv_step_plans_bytes: null pointer");
  *bytes = sizeof(StepPlans);
  return HV_OK;
}

int hv_step_set_option(int option, int value) {
  switch (option) {
    case HV_STEP_OPT_INFLIGHT:
      HV_REQUIRE(value >= 1 && value <= kMaxSlots, HV_E_INVALID,
                 "hv_step_set_option: in-flight copies %d outside [1, %d]", value, kMaxSlots);
      g_opt_inflight = value;
      return HV_OK;
    case HV_STEP_OPT_EVICT_FIRST:
      g_opt_evict_first = value != 0;
      return HV_OK;
    case HV_STEP_OPT_LOCAL_QKV_BARRIER:
      g_opt_local_qkv_barrier = value != 0;
      return HV_OK;
    case HV_STEP_OPT_REF_BLAS_RUNS:
      return set_ref_blas_runs(value);
    default:
      HV_REQUIRE(false, HV_E_INVALID, "hv_step_set_option: unknown option %d", option);
  }
}

int hv_step_launch(const hv_step_desc* desc, int flags, void* stream) {
  HV_REQUIRE(desc, HV_E_INVALID, "hv_step_launch: null descriptor");
  hv_step_desc h = *desc;
  HV_REQUIRE(h.head_dim == kHd, HV_E_UNSUPPORTED, "hv_step_launch: head_dim %d", h.head_dim);
  HV_REQUIRE(h.hidden % kBlock == 0 && h.ffn % kBlock == 0, HV_E_UNSUPPORTED,
             "hv_step_launch: hidden/ffn not multiples of 32");
  HV_REQUIRE(h.hidden <= kMaxHidden, HV_E_UNSUPPORTED, "hv_step_launch: hidden %d > %d",
             h.hidden, kMaxHidden);
  HV_REQUIRE(h.plans != nullptr, HV_E_INVALID, "hv_step_launch: plans not set (hv_step_plans)");
  HV_REQUIRE(h.n_layer > 0 && h.layers != nullptr, HV_E_INVALID,
             "hv_step_launch: no layer table");
  HV_REQUIRE(h.attn_chunks > 0 && h.attn_chunks <= kMaxFront &&
                 (h.attn_chunks & (h.attn_chunks - 1)) == 0,
             HV_E_INVALID, "hv_step_launch: attn_chunks %d (a power of two, at most %d)",
             h.attn_chunks, kMaxFront);
  const int gs = h.n_head / h.n_kv;
  HV_REQUIRE(gs == 1 || gs == 2 || gs == 4 || gs == 8, HV_E_UNSUPPORTED,
             "hv_step_launch: group size %d", gs);
  HV_REQUIRE(h.world >= 1 && h.world <= HV_MAX_WORLD && h.rank >= 0 && h.rank < h.world,
             HV_E_INVALID, "hv_step_launch: rank %d of world %d", h.rank, h.world);
  HV_REQUIRE(h.world == 1 || h.peers != nullptr, HV_E_INVALID,
             "hv_step_launch: a sharded step needs the peer table");
  HV_REQUIRE(h.hidden % (8 * h.world) == 0, HV_E_UNSUPPORTED,
             "hv_step_launch: hidden %d does not split into 8-row tiles over %d ranks",
             h.hidden, h.world);
  const int world = h.world;
  const int qdim = h.n_head * kHd * world, ffn_all = h.ffn * world;
  const int nslots =
      step_slots(gs, h.hidden, qdim, ffn_all, h.cap, h.attn_chunks, h.n_layer);
  HV_REQUIRE(nslots >= 4, HV_E_UNSUPPORTED,
             "hv_step_launch: shared memory leaves %d ring slots (need 4)", nslots);
  const StepLayout lay =
      step_layout(gs, h.hidden, qdim, ffn_all, h.cap, h.attn_chunks, nslots, h.n_layer);
  const size_t smem = lay.total;
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  {
    // multi-leaf GEMV rows meet in the work area: tiles per CTA x 8 rows x leaves
    const int nqkv = (h.n_head + 2 * h.n_kv) * kHd;
    const int hrows = h.hidden / world;
    const int tiles[5] = {pp_tiles(nqkv, 0), pp_tiles(hrows, 0), pp_tiles(2 * h.ffn, h.ffn),
                          pp_tiles(hrows, 0), pp_tiles(h.head_rows, 0)};
    const int ks[5] = {h.hidden, qdim, h.hidden, ffn_all, h.hidden};
    for (int i = 0; i < 5; ++i) {
      GvPlan gp;
      HV_REQUIRE(gv_make_plan(ks[i] / kBlock, &gp), HV_E_UNSUPPORTED,
                 "hv_step_launch: K = %d has too many pairwise leaves", ks[i]);
      // gate/up: whole units of 8 tiles per CTA, plus 4 staged SiLU outputs per tile
      const int per = i == 2 ? ((tiles[i] + 7) / 8 + sms - 1) / sms * 8 : (tiles[i] + sms - 1) / sms;
      const size_t need = (size_t)per * (8 * (gp.nleaf > 1 ? gp.nleaf : 0) + (i == 2 ? 4 : 0)) * 4;
      HV_REQUIRE(need <= lay.ring - lay.work, HV_E_UNSUPPORTED,
                 "hv_step_launch: %zu B of leaf values exceed the work area", need);
    }
  }
  HV_REQUIRE(h.kv_dtype == HV_KV_F32 || h.kv_dtype == HV_KV_F16, HV_E_INVALID,
             "hv_step_launch: kv_dtype %d (HV_KV_F32 or HV_KV_F16)", h.kv_dtype);
  HV_REQUIRE(h.w4_layout == HV_W4_PP || h.w4_layout == HV_W4_DQ, HV_E_INVALID,
             "hv_step_launch: w4_layout %d (HV_W4_PP or HV_W4_DQ)", h.w4_layout);
  const bool f16 = h.kv_dtype == HV_KV_F16;
  const int variant = h.w4_layout == HV_W4_DQ ? (f16 ? 4 : 3) : f16 ? 2 : 0;
  HV_REQUIRE(h.cap <= kExactMaxCap, HV_E_UNSUPPORTED, "hv_step_launch: cap %d > %d", h.cap,
             kExactMaxCap);
  HV_REQUIRE(h.n_kv * h.attn_chunks <= sms, HV_E_UNSUPPORTED,
             "hv_step_launch: %d kv heads x %d chunks need one CTA per attention item (%d)",
             h.n_kv, h.attn_chunks, sms);
  HV_REQUIRE(h.kv_base != nullptr && h.kv_rows >= (long long)2 * h.n_kv * h.cap &&
                 ((uintptr_t)h.kv_base & 15) == 0,
             HV_E_INVALID, "hv_step_launch: kv_base/kv_rows do not describe the KV cache");
  CUtensorMap vmap;
  rc = vslice_map(h.kv_base, h.kv_rows, f16 ? 2 : 4, kCtxRows, &vmap);
  if (rc) return rc;
  void* fn = step_fn(gs, variant);
  {
    // set the function's shared-memory limit once per (kernel, device, size)
    static std::mutex mu;
    static size_t done[20][64];
    int dev = 0;
    HV_CUDA(cudaGetDevice(&dev));
    const int gi = (gs == 1 ? 0 : gs == 2 ? 1 : gs == 4 ? 2 : 3) + 4 * variant;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || done[gi][dev] < smem) {
      HV_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      if (dev >= 0 && dev < 64) done[gi][dev] = smem;
    }
  }
  HV_REQUIRE((flags & ~(HV_STEP_HEAD | HV_STEP_ARGMAX)) == 0, HV_E_INVALID,
             "hv_step_launch: unknown flags 0x%x", flags);
  if (g_opt_local_qkv_barrier && world > 1) flags |= kFlagLocalQkvBarrier;

  int inflight = g_opt_inflight, evict_first = g_opt_evict_first, runs = ref_blas_runs();
  void* args[] = {(void*)&h, (void*)&flags, (void*)&nslots, (void*)&inflight,
                  (void*)&evict_first, (void*)&runs, (void*)&vmap};
  HV_CUDA(cudaLaunchCooperativeKernel(fn, dim3(sms), dim3(kStepThreads), args, smem,
                                      (cudaStream_t)stream));
  return HV_OK;
}

}  // extern "C"
