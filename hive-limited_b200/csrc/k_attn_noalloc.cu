// hv_attn_decode_noalloc: split-sequence decode attention whose scratch is a fixed,
// file-scope device array instead of memory the library allocates.
//
// Who needs it: a caller that cannot let the library call cudaMalloc/cudaFree. A
// serving process that hands all of HBM to its own weight + KV pool up front would see
// a surprise allocation fail; cudaFree synchronises the whole device and would stall
// every other stream of a latency-bound decode loop; and an allocation made while a
// foreign memory pool or allocator lock is held can deadlock or fragment that pool.
// hv_attn_decode grows its scratch with cudaMalloc on first use and whenever a larger
// cache is seen; this entry point never allocates.
//
// The scratch: kNaScratchBytes (2 MiB) of `static __device__` memory, shared by every
// call on a device. Its first 256 bytes are the per-kv-head completion tickets (must be
// zero when a call starts: each call clears them with cudaMemsetAsync on its stream);
// the rest holds the chunk partials (nkv * chunks * group * 132 floats). A problem whose
// partials do not fit, or with more than 64 kv heads, is rejected with HV_E_INVALID.
// Calls that overlap on the GPU (two streams, or two host threads on one device) share
// the same bytes and race: order them on one stream.
//
// Set-up, once per device, happens on the first call made with that device current: it
// takes the array's device address with cudaGetSymbolAddress and sets the kernels'
// shared-memory attribute (which also loads them). Make that first call before any
// stream capture.
#include <mutex>

#include "attn_decode.cuh"
#include "hv_internal.h"

namespace hv {
namespace {

constexpr size_t kNaScratchBytes = 2u << 20;
constexpr size_t kNaTicketBytes = 256;
constexpr int kNaMaxKv = (int)(kNaTicketBytes / sizeof(int));
constexpr int kNaThreads = 256;

static __device__ __align__(256) unsigned char g_na_scratch[kNaScratchBytes];

template <int GS>
__global__ void __launch_bounds__(kNaThreads) k_attn_na(const float* __restrict__ q,
                                                        const float* __restrict__ kc,
                                                        const float* __restrict__ vc,
                                                        float* __restrict__ ctx,
                                                        const float* __restrict__ scale_p,
                                                        const int32_t* __restrict__ pos_p,
                                                        int cap, int nch,
                                                        float* __restrict__ part,
                                                        int* __restrict__ ticket) {
  extern __shared__ __align__(16) float fsm[];
  const int nw = blockDim.x >> 5;
  float* q_s = fsm;
  float* lg_s = q_s + GS * kHd;
  float* red_s = lg_s + kAttnChunkMax * GS;
  float* stat_s = red_s + nw * GS * kHd;
  __shared__ int last;
  const int g = blockIdx.x / nch, c = blockIdx.x % nch;
  const int pos = *pos_p;
  for (int e = threadIdx.x; e < GS * kHd; e += blockDim.x) q_s[e] = q[(size_t)g * GS * kHd + e];
  __syncthreads();
  int t0, t1;
  chunk_bounds(pos + 1, nch, c, &t0, &t1);
  float* mypart = part + ((size_t)g * nch + c) * GS * kPartStride;
  attn_chunk<GS>(q_s, kc + (size_t)g * cap * kHd, vc + (size_t)g * cap * kHd, t0, t1,
                 *scale_p, pos, nullptr, nullptr, lg_s, red_s, stat_s, mypart);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(ticket + g, 1) == nch - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  attn_merge<GS>(part + (size_t)g * nch * GS * kPartStride, nch, ctx + (size_t)g * GS * kHd,
                 red_s);
}

struct NaDevice {
  std::once_flag once;
  int rc = HV_OK;
  unsigned char* base = nullptr;
};
static NaDevice g_na[64];

template <int GS>
static cudaError_t na_attr() {
  return cudaFuncSetAttribute((const void*)k_attn_na<GS>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)attn_smem_bytes<GS>(kNaThreads / 32));
}

static int na_setup(NaDevice* d) {
  void* p = nullptr;
  HV_CUDA(cudaGetSymbolAddress(&p, g_na_scratch));
  HV_REQUIRE(p != nullptr && ((uintptr_t)p & 255u) == 0, HV_E_UNSUPPORTED,
             "hv_attn_decode_noalloc: scratch address %p is not 256-byte aligned", p);
  HV_CUDA(na_attr<1>());
  HV_CUDA(na_attr<2>());
  HV_CUDA(na_attr<4>());
  HV_CUDA(na_attr<8>());
  d->base = (unsigned char*)p;
  return HV_OK;
}

// The chunk count of hv_attn_decode (so both entry points split the sequence alike).
static int na_chunks(int nkv, int cap, int* out) {
  int sms = 0;
  const int rc = sm_count(&sms);
  if (rc) return rc;
  const int nch = (sms + nkv - 1) / nkv;
  const int need = (cap + kAttnChunkMax - 1) / kAttnChunkMax;
  *out = nch > need ? nch : need;
  return HV_OK;
}

template <int GS>
static int na_launch(const float* q, const float* kc, const float* vc, float* ctx,
                     const float* scale, const int32_t* pos, int nkv, int cap, int nch,
                     float* part, int* ticket, cudaStream_t st) {
  const size_t smem = attn_smem_bytes<GS>(kNaThreads / 32);
  k_attn_na<GS><<<nkv * nch, kNaThreads, smem, st>>>(q, kc, vc, ctx, scale, pos, cap, nch,
                                                     part, ticket);
  HV_LAUNCHED("k_attn_na");
}

}  // namespace
}  // namespace hv

using namespace hv;

extern "C" int hv_attn_decode_noalloc(const float* q, const float* kc, const float* vc,
                                      float* ctx, const float* scale, const int32_t* pos,
                                      int nq, int hd, int group, int kvstride, void* stream) {
  HV_REQUIRE(q && kc && vc && ctx && scale && pos && nq > 0 && group > 0 && kvstride > 0,
             HV_E_INVALID, "hv_attn_decode_noalloc: bad arguments");
  HV_REQUIRE(hd == kHd, HV_E_UNSUPPORTED, "hv_attn_decode_noalloc: head_dim %d (only 128)", hd);
  HV_REQUIRE(nq % group == 0 && kvstride % hd == 0, HV_E_INVALID,
             "hv_attn_decode_noalloc: nq %% group or kvstride %% hd is not zero");
  HV_REQUIRE(group == 1 || group == 2 || group == 4 || group == 8, HV_E_UNSUPPORTED,
             "hv_attn_decode_noalloc: group size %d (1, 2, 4 or 8)", group);
  const int nkv = nq / group, cap = kvstride / hd;
  HV_REQUIRE(nkv <= kNaMaxKv, HV_E_INVALID,
             "hv_attn_decode_noalloc: %d kv heads exceed the fixed scratch's limit of %d", nkv,
             kNaMaxKv);
  int nch = 0;
  int rc = na_chunks(nkv, cap, &nch);
  if (rc) return rc;
  const size_t part_bytes = (size_t)nkv * nch * group * kPartStride * sizeof(float);
  HV_REQUIRE(part_bytes <= kNaScratchBytes - kNaTicketBytes, HV_E_INVALID,
             "hv_attn_decode_noalloc: %zu bytes of partial softmax state (%d kv heads x %d "
             "chunks x group %d) exceed the fixed scratch of %zu bytes",
             part_bytes, nkv, nch, group, kNaScratchBytes - kNaTicketBytes);
  HV_REQUIRE(nch <= kAttnMaxChunks, HV_E_UNSUPPORTED,
             "hv_attn_decode_noalloc: %d chunks per kv head (at most %d)", nch, kAttnMaxChunks);

  int dev = 0;
  HV_CUDA(cudaGetDevice(&dev));
  HV_REQUIRE(dev >= 0 && dev < 64, HV_E_UNSUPPORTED, "device index %d out of range", dev);
  NaDevice& d = g_na[dev];
  std::call_once(d.once, [&d] { d.rc = na_setup(&d); });
  if (d.rc) {
    set_error("hv_attn_decode_noalloc: set-up on device %d failed (status %d)", dev, d.rc);
    return d.rc;
  }
  int* ticket = (int*)d.base;
  float* part = (float*)(d.base + kNaTicketBytes);
  cudaStream_t st = (cudaStream_t)stream;
  HV_CUDA(cudaMemsetAsync(ticket, 0, (size_t)nkv * sizeof(int), st));
  switch (group) {
    case 1: return na_launch<1>(q, kc, vc, ctx, scale, pos, nkv, cap, nch, part, ticket, st);
    case 2: return na_launch<2>(q, kc, vc, ctx, scale, pos, nkv, cap, nch, part, ticket, st);
    case 4: return na_launch<4>(q, kc, vc, ctx, scale, pos, nkv, cap, nch, part, ticket, st);
    default: return na_launch<8>(q, kc, vc, ctx, scale, pos, nkv, cap, nch, part, ticket, st);
  }
}
