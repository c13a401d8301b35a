// hv_attn_decode_noalloc: the decode attention of hv_attn_decode whose scratch is a
// fixed, file-scope device array instead of memory the library allocates.
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
// call on a device: the scores [nq][cap] and the chunk maxima [nq][chunks] that the
// context kernel reads (nq x (cap + chunks) floats). Every call writes all of it that it
// reads, so nothing has to start at zero. A problem that does not fit is rejected with
// HV_E_INVALID. Calls that overlap on the GPU (two streams, or two host threads on one
// device) share the same bytes and race: order them on one stream.
//
// Set-up, once per device, happens on the first call made with that device current: it
// takes the array's device address with cudaGetSymbolAddress. Make that first call
// before any stream capture.
#include <mutex>

#include "attn_decode.cuh"
#include "hv_internal.h"

namespace hv {
namespace {

constexpr size_t kNaScratchBytes = 2u << 20;

static __device__ __align__(256) unsigned char g_na_scratch[kNaScratchBytes];

struct NaDevice {
  std::once_flag once;
  int rc = HV_OK;
  float* base = nullptr;
};
static NaDevice g_na[64];

static int na_setup(NaDevice* d) {
  void* p = nullptr;
  HV_CUDA(cudaGetSymbolAddress(&p, g_na_scratch));
  HV_REQUIRE(p != nullptr && ((uintptr_t)p & 255u) == 0, HV_E_UNSUPPORTED,
             "hv_attn_decode_noalloc: scratch address %p is not 256-byte aligned", p);
  d->base = (float*)p;
  return HV_OK;
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
  int nch = 0;
  int rc = attn_exact_chunks(nkv, cap, &nch);
  if (rc) return rc;
  const size_t need = attn_exact_scratch_floats(nq, cap, nch) * sizeof(float);
  HV_REQUIRE(need <= kNaScratchBytes, HV_E_INVALID,
             "hv_attn_decode_noalloc: %zu bytes of scores and chunk maxima (%d heads x (%d "
             "positions + %d chunks)) exceed the fixed scratch of %zu bytes",
             need, nq, cap, nch, kNaScratchBytes);

  int dev = 0;
  HV_CUDA(cudaGetDevice(&dev));
  HV_REQUIRE(dev >= 0 && dev < 64, HV_E_UNSUPPORTED, "device index %d out of range", dev);
  NaDevice& d = g_na[dev];
  std::call_once(d.once, [&d] { d.rc = na_setup(&d); });
  if (d.rc) {
    set_error("hv_attn_decode_noalloc: set-up on device %d failed (status %d)", dev, d.rc);
    return d.rc;
  }
  return attn_exact_launch(group, false, q, 0, kc, vc, ctx, 0, scale, pos, 0, nq, cap, nch, 1,
                           d.base, 0, (cudaStream_t)stream);
}
