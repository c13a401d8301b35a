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
// tiles of every GEMV, the K and V rows of its attention chunks, its rows of the LM head
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
//   P2 attn : per (kv head, chunk): q/k norm + RoPE, KV append at pos, split softmax;
//             last CTA of each kv head merges                     -> ctx
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

#include <cuda_fp16.h>

#include "attn_decode.cuh"
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

// Run-time tunables (hv_step_set_option): bulk copies a producer keeps in flight, and
// whether streamed bytes are marked evict-first in L2. Copies beyond what saturates HBM
// only queue in front of the consumers' own (latency-critical) loads.
static int g_opt_inflight = 6;
static int g_opt_evict_first = 1;
static int g_opt_local_qkv_barrier = 0;
static int g_opt_split_merge = 0;
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
  unsigned phase;                // top bit of the grid barrier counter to wait for next
  unsigned xphase;               // sharded: top bit of the cross-rank counter (CTA 0)
  unsigned gen;                  // sharded: generation of the local release word
  unsigned long long wait[kConsWarps];   // ns each consumer warp waited for ring slots
  long long busy[kConsWarps];            // cycles spent computing attention scores
};

// Byte offsets of the dynamic shared memory regions (host and device agree).
struct StepLayout {
  size_t layers, bars, act_q, act_sb, work, ring, total;
};

HV_HD size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

HV_HD size_t attn_area_floats(int gs, int cap, int nch) {
  const size_t chunk_max = ((size_t)cap + nch - 1) / nch;
  const size_t lg = ((size_t)chunk_max * gs + 3) & ~size_t(3);
  return (size_t)gs * kHd + 2 * kHd + (size_t)(gs + 1) * kHd + 4 * (size_t)gs + lg +
         (size_t)kConsWarps * gs * kHd;
}

HV_HD StepLayout step_layout(int gs, int hid, int qdim, int ffn, int cap, int nch, int nslots,
                             int n_layer) {
  const int kmax = hid > qdim ? (hid > ffn ? hid : ffn) : (qdim > ffn ? qdim : ffn);
  StepLayout L;
  L.layers = align_up(sizeof(StepShared), 16);
  L.bars = L.layers + align_up((size_t)n_layer * sizeof(hv_layer_w), 16);
  L.act_q = L.bars + 2 * kMaxSlots * sizeof(uint64_t);
  L.act_sb = L.act_q + align_up((size_t)kmax, 16);
  L.work = L.act_sb + align_up((size_t)(kmax / kBlock) * 8, 16);
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

// Positions [t0, t1) of attention chunk c, and te: rows [t0, te) come from the cache,
// row pos (if in the chunk) from this step's qkv.
HV_DEV void attn_rows(int pos, int nch, int c, int* t0, int* t1, int* te) {
  chunk_bounds(pos + 1, nch, c, t0, t1);
  *te = max(*t0, min(*t1, pos));
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

  // Claims the next slot (waiting until its previous contents were released and until
  // fewer than `inflight` earlier copies are still in flight) and starts up to two
  // copies into it.
  HV_DEV void issue(const void* a, unsigned na, const void* b, unsigned nb_, unsigned b_off) {
    if (!live) return;
    if (q >= (unsigned)R.ns && !mbar_probe(R.empty_of(q), R.parity(q) ^ 1u)) {
      const unsigned long long t0 = global_ns();
      if (!mbar_wait(R.empty_of(q), R.parity(q) ^ 1u, S, status, kProducerWaitNs)) {
        live = false;
        return;
      }
      t_empty += global_ns() - t0;
    }
    if (q >= inflight) {
      const unsigned p = q - inflight;
      if (!mbar_probe(R.full_of(p), R.parity(p))) {
        const unsigned long long t0 = global_ns();
        if (!mbar_wait(R.full_of(p), R.parity(p), S, status, kProducerWaitNs)) {
          live = false;
          return;
        }
        t_flight += global_ns() - t0;
      }
    }
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

  // K rows then V rows [t0, te) of kv head g for one attention work item (KT: the
  // cache's element type, float or __half).
  template <class KT>
  HV_DEV void kv(const KT* kc, const KT* vc, int g, int cap, int t0, int te) {
    for (int pass = 0; pass < 2; ++pass) {
      const KT* base = (pass == 0 ? kc : vc) + (size_t)g * cap * kHd;
      for (int r = t0; r < te && live; r += kSlotRows) {
        const unsigned n = (unsigned)min(kSlotRows, te - r);
        issue(base + (size_t)r * kHd, n * kHd * (unsigned)sizeof(KT), nullptr, 0, 0);
      }
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

template <class KT>
HV_DEV void produce(const hv_step_desc& D, const hv_layer_w* Ls, int flags, int pos,
                    const Ring& R, StepShared& S, int inflight, int evict_first) {
  Producer P(R, S, D.status, inflight, evict_first);
  const int world = D.world > 1 ? D.world : 1;
  const int hid = D.hidden, ffn = D.ffn, qdim = D.n_head * kHd * world, hrows = hid / world;
  const int nqkv = (D.n_head + 2 * D.n_kv) * kHd;
  const int nch = D.attn_chunks;
  const int it_hid = pp_iters(hid / kBlock), it_q = pp_iters(qdim / kBlock),
            it_ffn = pp_iters(ffn * world / kBlock);
  int off = 0, t0, t1;
  for (int l = 0; l < D.n_layer && P.live; ++l) {
    const hv_layer_w* L = Ls + l;
    phase_tiles(pp_tiles(nqkv, 0), &off, &t0, &t1);
    P.gemv(L->qkv_b4, L->qkv_sw, it_hid, t0, t1, S.P.gv_hid.nleaf);
    for (int wi = blockIdx.x; wi < D.n_kv * nch; wi += gridDim.x) {
      int a0, a1, ae;
      attn_rows(pos, nch, wi % nch, &a0, &a1, &ae);
      P.kv(reinterpret_cast<const KT*>(L->kc), reinterpret_cast<const KT*>(L->vc), wi / nch,
           D.cap, a0, ae);
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

// ---- attention -------------------------------------------------------------------------

// Rows per score group: enough that one butterfly reduces 32 values (4 rows for GS = 8).
// Each score is the lane-partial dot (x*x, then three fma) summed over the 32 lanes with
// the xor-16, 8, 4, 2, 1 tree whatever the group size, so the grouping changes no bit.
template <int GS>
constexpr int kScoreRows = GS >= 8 ? 4 : 8;

// Rows tb .. tb + RW - 1 of a block whose cached rows [r0, te) sit in `slot` (null for a
// block that holds only pos): one shared-memory load per cached row (index clamped inside
// the slot, so no branch precedes it), the pos row loaded once if this group holds it,
// rows from `tend` on (not this block's) and stale slot rows selected to zero.
// Dims 4 lane .. 4 lane + 3 of row r of a ring slot of cache rows, as floats (half ->
// float is exact).
HV_DEV float4 slot_row4(const float*, unsigned slot, int r, int lane) {
  return lds_f4(slot + (unsigned)(r * kHd + 4 * lane) * 4);
}
HV_DEV float4 slot_row4(const __half*, unsigned slot, int r, int lane) {
  const uint2 w = lds_u2(slot + (unsigned)(r * kHd + 4 * lane) * 2);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <int RW, class KT>
HV_DEV void block_rows(float4 (&kv)[RW], int tb, int tend, int te, int pos, unsigned slot,
                       int r0, unsigned pos_s, int lane) {
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int p = 0; p < RW; ++p) {
    const int r = min(tb + p - r0, kSlotRows - 1);
    kv[p] = slot ? slot_row4(static_cast<const KT*>(nullptr), slot, r, lane) : zero;
  }
  const bool has_pos = pos >= tb && pos < tb + RW && pos < tend && pos >= te;
  const float4 pv = has_pos ? lds_f4(pos_s + 16 * lane) : zero;
#pragma unroll
  for (int p = 0; p < RW; ++p) {
    const int t = tb + p;
    kv[p] = (t < te && t < tend) ? kv[p] : ((has_pos && t == pos) ? pv : zero);
  }
}

// Scores of positions tb .. tb + kScoreRows - 1 (those below tend) for the GS heads, the
// arithmetic of attn_chunk in attn_decode.cuh. slot (0: none), kpos_s and lg_s are shared
// addresses.
template <int GS, class KT>
HV_DEV void group_scores(const float4 (&qv)[GS], int tb, int tend, int t0, int te, int pos,
                         unsigned slot, int r0, unsigned kpos_s, float scale, unsigned lg_s) {
  constexpr int RW = kScoreRows<GS>;
  const int lane = threadIdx.x & 31;
  float4 kv[RW];
  block_rows<RW, KT>(kv, tb, tend, te, pos, slot, r0, kpos_s, lane);
  float v[RW * GS];
#pragma unroll
  for (int p = 0; p < RW; ++p)
#pragma unroll
    for (int i = 0; i < GS; ++i) {
      float s = qv[i].x * kv[p].x;
      s = fmaf(qv[i].y, kv[p].y, s);
      s = fmaf(qv[i].z, kv[p].z, s);
      s = fmaf(qv[i].w, kv[p].w, s);
      v[p * GS + i] = s;
    }
  int idx;
  const float tot = halving_reduce<RW * GS>(v, lane, &idx);
  constexpr int dup = 32 / (RW * GS) > 0 ? 32 / (RW * GS) : 1;
  if ((lane & (dup - 1)) == 0) {
    const int p = idx / GS, i = idx % GS;
    const int t = tb + p;
    if (t < tend) {
      const float val = tot * scale;
      asm volatile("st.shared.f32 [%0], %1;" :: "r"(lg_s + (unsigned)((t - t0) * GS + i) * 4),
                   "f"(val) : "memory");
    }
  }
}

// Probability-weighted V rows [tb, tb + 8) (those below tend) into acc, rows in order
// (the order of attn_chunk); all loads are issued before the first multiply-add.
template <int GS, class KT>
HV_DEV void group_values(float4 (&acc)[GS], int tb, int tend, int t0, int te, int pos,
                         unsigned slot, int r0, unsigned vpos_s, unsigned lg_s) {
  constexpr int RW = 8;
  const int lane = threadIdx.x & 31;
  float4 vv[RW];
  float w[RW][GS];
  block_rows<RW, KT>(vv, tb, tend, te, pos, slot, r0, vpos_s, lane);
#pragma unroll
  for (int p = 0; p < RW; ++p)
#pragma unroll
    for (int i = 0; i < GS; ++i)
      w[p][i] = (tb + p < tend) ? lds_f1(lg_s + (unsigned)((tb + p - t0) * GS + i) * 4) : 0.f;
#pragma unroll
  for (int p = 0; p < RW; ++p) {
    if (tb + p < tend) {
#pragma unroll
      for (int i = 0; i < GS; ++i) {
        acc[i].x = fmaf(w[p][i], vv[p].x, acc[i].x);
        acc[i].y = fmaf(w[p][i], vv[p].y, acc[i].y);
        acc[i].z = fmaf(w[p][i], vv[p].z, acc[i].z);
        acc[i].w = fmaf(w[p][i], vv[p].w, acc[i].w);
      }
    }
  }
}

// The attention phase: this CTA's (kv head, chunk) work items, K and V rows streamed
// through the ring (sequence numbers from *q). Same arithmetic, in the same order, as
// attn_chunk with eight warps (k_attn): blocks of 20 positions go to warp (block % 8)
// for the scores and the weighted V sum; warp i takes head i for the max and exp.
// KT = __half: the compressed-KV lane. This step's k and v rows are rounded to binary16
// before use, so row pos enters the scores and the V sum exactly as the appended cache
// row does (hv_kv_append_f16 then hv_attn_decode_f16).
template <int GS, bool kSplitMerge, class KT>
__device__ __noinline__ void attn_ring(const hv_step_desc& D, const hv_layer_w* L, int pos,
                                       const Ring R, unsigned* qp, StepShared& S,
                                       float* area, int tb) {
  const int nkv = D.n_kv, nch = D.attn_chunks, cap = D.cap, nq = D.n_head;
  const int chunk_max = (cap + nch - 1) / nch;
  const int lg_floats = (chunk_max * GS + 3) & ~3;   // keeps red_s 16-byte aligned
  float* q_s = area;
  float* kpos_s = q_s + GS * kHd;
  float* vpos_s = kpos_s + kHd;
  float* tmp_s = vpos_s + kHd;                       // (GS + 1) x 128
  float* stat_s = tmp_s + (GS + 1) * kHd;            // 2 GS (+pad)
  float* lg_s = stat_s + 4 * GS;
  float* red_s = lg_s + lg_floats;                   // accessed as float4
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* cs = D.cos_t + (size_t)pos * (kHd / 2);
  const float* sn = D.sin_t + (size_t)pos * (kHd / 2);
  const float scale = D.attn_scale;
  for (int wi = blockIdx.x; wi < nkv * nch; wi += gridDim.x) {
    const int g = wi / nch, c = wi % nch;
    int t0, t1, te;
    attn_rows(pos, nch, c, &t0, &t1, &te);
    const int n = t1 - t0;
    const int nk = (te - t0 + kSlotRows - 1) / kSlotRows;
    const unsigned qk = *qp, qv0 = *qp + (unsigned)nk;
    *qp += 2u * (unsigned)nk;
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
    csync();
    trace_mark(D, tb + 14);
    trace_wait(D, S, tb + 20);
    if (c == nch - 1 && threadIdx.x < kHd) {         // the chunk holding pos appends
      KT* kc = reinterpret_cast<KT*>(L->kc) + (size_t)g * cap * kHd;
      KT* vc = reinterpret_cast<KT*>(L->vc) + (size_t)g * cap * kHd;
      kc[(size_t)pos * kHd + threadIdx.x] = to_kv<KT>(kpos_s[threadIdx.x]);
      vc[(size_t)pos * kHd + threadIdx.x] = to_kv<KT>(vpos_s[threadIdx.x]);
    }

    // ---- scores: block m = positions [t0 + 20 m, +20) (one ring slot of K rows, row
    // pos from kpos_s) to warp m % 8, so each slot has a single consumer warp; the block
    // after the last slot holds only pos when pos starts a block
    float4 qv[GS];
#pragma unroll
    for (int i = 0; i < GS; ++i) qv[i] = reinterpret_cast<const float4*>(q_s + i * kHd)[lane];
    bool ok = true;
    const int nblk = (n + kSlotRows - 1) / kSlotRows;
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
      for (int tg = r0; tg < r1; tg += kScoreRows<GS>)
        group_scores<GS, KT>(qv, tg, r1, t0, te, pos, slot, r0, sh_addr(kpos_s), scale,
                             sh_addr(lg_s));
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

    // ---- per-head max and exp: warp i handles head i
    for (int i = warp; i < GS; i += kConsWarps) {
      float mx = -INFINITY;
      for (int t = lane; t < n; t += 32) mx = fmaxf(mx, lg_s[t * GS + i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
      float l = 0.f;
      for (int t = lane; t < n; t += 32) {
        const float e = (n > 0) ? expf(lg_s[t * GS + i] - mx) : 0.f;
        lg_s[t * GS + i] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
      if (lane == 0) { stat_s[2 * i] = mx; stat_s[2 * i + 1] = l; }
    }
    csync();
    trace_mark(D, tb + 16);
    trace_wait(D, S, tb + 20);

    // ---- probability-weighted V sum: V rows from the ring, the same block -> warp map,
    // positions in order within a block
    float4 acc[GS];
#pragma unroll
    for (int i = 0; i < GS; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int m = warp; m < nblk && ok; m += kConsWarps) {
      const int r0 = t0 + m * kSlotRows, r1 = min(r0 + kSlotRows, t1);
      unsigned slot = 0;
      if (m < nk) {
        const unsigned q = qv0 + (unsigned)m;
        ok = warp_wait(R.full_of(q), R.parity(q), S, D.status);
        if (!ok) break;
        slot = sh_addr(R.slot(q));
      }
      for (int tg = r0; tg < r1; tg += 8)
        group_values<GS, KT>(acc, tg, r1, t0, te, pos, slot, r0, sh_addr(vpos_s),
                             sh_addr(lg_s));
      if (m < nk) {
        __syncwarp();
        if (lane == 0) mbar_arrive_n(R.empty_of(qv0 + (unsigned)m), kConsWarps);
      }
    }
#pragma unroll
    for (int i = 0; i < GS; ++i)
      reinterpret_cast<float4*>(red_s + ((size_t)warp * GS + i) * kHd)[lane] = acc[i];
    csync();
    float* part = D.part + ((size_t)g * nch + c) * GS * kPartStride;
    for (int e = threadIdx.x; e < GS * kHd; e += kConsThreads) {
      float s = 0.f;
      for (int w = 0; w < kConsWarps; ++w) s += red_s[(size_t)w * GS * kHd + e];
      const int i = e / kHd, d = e % kHd;
      part[i * kPartStride + 4 + d] = s;
    }
    if (threadIdx.x < GS) {
      part[threadIdx.x * kPartStride + 0] = (n > 0) ? stat_s[2 * threadIdx.x] : -INFINITY;
      part[threadIdx.x * kPartStride + 1] = (n > 0) ? stat_s[2 * threadIdx.x + 1] : 0.f;
    }
    if constexpr (!kSplitMerge) __threadfence();
    csync();
    trace_mark(D, tb + 17);
    trace_wait(D, S, tb + 22);
    if constexpr (kSplitMerge) continue;             // merged after the grid barrier
    if (threadIdx.x == 0) S.flag = (atomicAdd(D.ticket + g, 1) == nch - 1);
    csync();
    trace_mark(D, tb + 18);
    if (S.flag) {
      __threadfence();
      // the o projection's input, quantised here: int8 [qdim] then (scale, sum) pairs;
      // this rank's heads start at head rank * n_head of the whole vector
      const int world = D.world > 1 ? D.world : 1, rank = world > 1 ? D.rank : 0;
      const int qall = nq * kHd * world, first = (rank * nq + g * GS) * kHd;
      int8_t* cq = reinterpret_cast<int8_t*>(D.ctx);
      int2* csb = reinterpret_cast<int2*>(cq + qall);
      attn_merge<GS, CSync, true>(D.part + (size_t)g * nch * GS * kPartStride, nch, nullptr,
                                  red_s, cq + first, csb + first / kBlock);
      if (threadIdx.x == 0) D.ticket[g] = 0;
      if (world > 1) {
        csync();
        share_bytes(D.peers->ctx, rank, world, cq, first, GS * kHd, qall);
      }
    }
    csync();
    trace_mark(D, tb + 19);
  }
}

// The attention merge as its own phase (HV_STEP_OPT_SPLIT_MERGE, one GPU): after the
// barrier that ends attention, each 32-value quantisation block of ctx is merged by one
// warp (blocks spread over the CTAs), instead of each kv head's whole merge by the last
// CTA of that head while every other CTA waits. Lane d of the warp does dim d of the
// block; the arithmetic and its order are attn_merge's (M = max_c m_c, w_c = exp(m_c - M),
// L = fma(w_c, l_c, L) and o = fma(w_c, acc_c, o) in chunk order, ctx = o * (1 / L), then
// quant_a8s of the block), so the bits are the same; only the loads are arranged for
// fewer L2 round trips. `area`: kConsWarps * nch floats.
template <int GS>
__device__ __noinline__ void merge_blocks(const hv_step_desc& D, float* area) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = D.n_head, nch = D.attn_chunks;
  constexpr int kPerHead = kHd / kBlock;
  const int nblk = nq * kPerHead;
  int8_t* cq = reinterpret_cast<int8_t*>(D.ctx);
  int2* csb = reinterpret_cast<int2*>(cq + (size_t)nq * kHd);
  float* wv = area + (size_t)warp * nch;
  for (int qb = blockIdx.x + warp * gridDim.x; qb < nblk; qb += gridDim.x * kConsWarps) {
    const int h = qb / kPerHead, d = (qb % kPerHead) * kBlock + lane;
    const int g = h / GS, i = h % GS;
    const float* ph = D.part + (size_t)g * nch * GS * kPartStride + (size_t)i * kPartStride;
    constexpr size_t kChunk = (size_t)GS * kPartStride;
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) M = fmaxf(M, __ldcg(ph + c * kChunk));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    // w_c = exp(m_c - M) and l_c, loaded by lane c of each pass of 32 chunks together (one
    // L2 round trip per pass); every lane then runs the chain L = fma(w_c, l_c, L) in chunk
    // order from shuffles, so L is attn_merge's value in every lane
    float L = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 32) {
      const int c = c0 + lane;
      float w = 0.f, l = 0.f;
      if (c < nch) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(ph + c * kChunk));
        w = expf(ml.x - M);
        l = ml.y;
        wv[c] = w;
      }
      const int n = min(32, nch - c0);
      for (int k = 0; k < n; ++k)
        L = fmaf(__shfl_sync(0xFFFFFFFFu, w, k), __shfl_sync(0xFFFFFFFFu, l, k), L);
    }
    const float inv = 1.0f / L;
    __syncwarp();                                   // wv[] of every lane
    float o = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 16) {
      float a[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) a[k] = (c0 + k < nch) ? __ldcg(ph + (c0 + k) * kChunk + 4 + d) : 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (c0 + k < nch) o = fmaf(wv[c0 + k], a[k], o);
    }
    int8_t q8;
    float sc;
    int bs;
    quant_block_warp(o * inv, lane, &q8, &sc, &bs);
    cq[(size_t)h * kHd + d] = q8;
    if (lane == 0) csb[qb] = make_int2(__float_as_int(sc), bs);
    __syncwarp();                                   // wv is reused by the next block
  }
}

// ---- the kernel ------------------------------------------------------------------------

template <int GS, bool kSplitMerge, class KT, bool kDq>
__global__ void __launch_bounds__(kStepThreads, 1) k_step(const hv_step_desc D, int flags,
                                                          int nslots, int inflight,
                                                          int evict_first) {
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
  __syncthreads();
  if (pos < 0 || pos >= D.cap || tok < 0 || tok >= D.vocab) {
    // every CTA reads the same values, so all leave here, before any copy or barrier
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(D.status, HV_E_INVALID);
    return;
  }
  if (threadIdx.x >= kConsThreads) {               // the producer warp: one lane copies
    if (threadIdx.x == kConsThreads)
      produce<KT>(D, Ls, flags, pos, R, S, inflight, evict_first);
    return;
  }

  // ---- consumers
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
    // P2: attention
    attn_ring<GS, kSplitMerge, KT>(D, L, pos, R, &q, S, work, tb);
    trace_mark(D, tb + 3);
    if (!grid_sync(D, S)) return;
    if constexpr (kSplitMerge) {
      merge_blocks<GS>(D, work);
      if (!grid_sync(D, S)) return;
    }
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
      S.flag = (atomicAdd(D.ticket + D.n_kv, 1) == (int)gridDim.x - 1);
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
      D.ticket[D.n_kv] = 0;
    }
  }
  trace_mark(D, th + 2);
}

// The step kernel for group size gs: variant 0 = f32 cache, 1 = f32 cache with the split
// merge, 2 = binary16 cache, 3 = f32 cache over dq weight tiles, 4 = binary16 cache over
// dq weight tiles.
static void* step_fn(int gs, int variant) {
  if (variant == 1) {
    switch (gs) {
      case 1: return (void*)k_step<1, true, float, false>;
      case 2: return (void*)k_step<2, true, float, false>;
      case 4: return (void*)k_step<4, true, float, false>;
      default: return (void*)k_step<8, true, float, false>;
    }
  }
  if (variant == 2) {
    switch (gs) {
      case 1: return (void*)k_step<1, false, __half, false>;
      case 2: return (void*)k_step<2, false, __half, false>;
      case 4: return (void*)k_step<4, false, __half, false>;
      default: return (void*)k_step<8, false, __half, false>;
    }
  }
  if (variant == 3) {
    switch (gs) {
      case 1: return (void*)k_step<1, false, float, true>;
      case 2: return (void*)k_step<2, false, float, true>;
      case 4: return (void*)k_step<4, false, float, true>;
      default: return (void*)k_step<8, false, float, true>;
    }
  }
  if (variant == 4) {
    switch (gs) {
      case 1: return (void*)k_step<1, false, __half, true>;
      case 2: return (void*)k_step<2, false, __half, true>;
      case 4: return (void*)k_step<4, false, __half, true>;
      default: return (void*)k_step<8, false, __half, true>;
    }
  }
  switch (gs) {
    case 1: return (void*)k_step<1, false, float, false>;
    case 2: return (void*)k_step<2, false, float, false>;
    case 4: return (void*)k_step<4, false, float, false>;
    default: return (void*)k_step<8, false, float, false>;
  }
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
  int nch = sms / n_kv;
  if (nch < 1) nch = 1;
  const int need = (cap + 511) / 512;
  if (nch < need) nch = need;
  HV_REQUIRE(nch <= kAttnMaxChunks, HV_E_UNSUPPORTED,
             "hv_step_config: %d attention chunks per kv head (at most %d; cap %d is too long)",
             nch, kAttnMaxChunks, cap);
  *chunks = nch;
  *part_floats = (size_t)n_kv * nch * group * kPartStride;
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
    case HV_STEP_OPT_SPLIT_MERGE:
      g_opt_split_merge = value != 0;
      return HV_OK;
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
  HV_REQUIRE(h.attn_chunks > 0 && 2 * h.attn_chunks + 1 <= kConsWarps * kHd, HV_E_INVALID,
             "hv_step_launch: attn_chunks %d outside [1, %d]", h.attn_chunks,
             (kConsWarps * kHd - 1) / 2);
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
  // the split merge (one GPU, f32 cache): its per-warp chunk weights live in the work area
  const bool split_merge = g_opt_split_merge && world == 1 && h.kv_dtype == HV_KV_F32 &&
      h.w4_layout == HV_W4_PP &&
      (lay.ring - lay.work) / sizeof(float) >= (size_t)kConsWarps * h.attn_chunks;
  const bool f16 = h.kv_dtype == HV_KV_F16;
  const int variant = h.w4_layout == HV_W4_DQ ? (f16 ? 4 : 3) : f16 ? 2 : split_merge ? 1 : 0;
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

  int inflight = g_opt_inflight, evict_first = g_opt_evict_first;
  void* args[] = {(void*)&h, (void*)&flags, (void*)&nslots, (void*)&inflight,
                  (void*)&evict_first};
  HV_CUDA(cudaLaunchCooperativeKernel(fn, dim3(sms), dim3(kStepThreads), args, smem,
                                      (cudaStream_t)stream));
  return HV_OK;
}

}  // extern "C"
