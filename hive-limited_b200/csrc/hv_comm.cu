// The all-gather of the column-parallel layout on the C ABI: hv_comm_init /
// hv_comm_init_rank, hv_allgather, hv_comm_destroy.
//
// The fused step exchanges its activation slices itself (peer stores inside k_step).
// These entry points give every other caller -- a sharded LM head, an external engine,
// the tests -- the same exchange as a plain collective: each rank contributes `bytes`
// from its send buffer and every rank receives all ranks' contributions, rank after rank
// (the layout the sharded kernels produce: rank r owns a contiguous slice). NCCL carries
// it over NVLink / NVSwitch.
//
// Two ways to build a communicator: one process driving `ndev` GPUs (hv_comm_init, one
// NCCL communicator per device, calls grouped), or one process per GPU (hv_comm_init_rank
// with an id made once by hv_comm_unique_id and handed to every rank by the caller).
// Errors come back as status codes with hv_last_error set; nothing aborts.
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <new>

#include "hv_internal.h"

struct hv_comm {
  int ndev;                       // devices this process drives in the communicator
  int nranks;                     // ranks of the whole communicator
  int devs[HV_MAX_WORLD];
  ncclComm_t comms[HV_MAX_WORLD];
};

namespace hv {
namespace {

int nccl_fail(const char* what, ncclResult_t r) {
  set_error("%s: %s", what, ncclGetErrorString(r));
  return HV_E_COMM;
}

#define HV_NCCL(call)                                        \
  do {                                                       \
    ncclResult_t _r = (call);                                \
    if (_r != ncclSuccess) return nccl_fail(#call, _r);      \
  } while (0)

}  // namespace
}  // namespace hv

using namespace hv;

static_assert(sizeof(ncclUniqueId) <= HV_COMM_ID_BYTES, "NCCL id fits the ABI's id buffer");

extern "C" {

int hv_comm_unique_id(void* id_out) {
  HV_REQUIRE(id_out, HV_E_INVALID, "hv_comm_unique_id: null buffer");
  ncclUniqueId id;
  HV_NCCL(ncclGetUniqueId(&id));
  memset(id_out, 0, HV_COMM_ID_BYTES);
  memcpy(id_out, &id, sizeof(id));
  return HV_OK;
}

int hv_comm_init(int ndev, const int* devs, hv_comm** out) {
  HV_REQUIRE(out && devs && ndev >= 1 && ndev <= HV_MAX_WORLD, HV_E_INVALID,
             "hv_comm_init: %d devices (1..%d)", ndev, HV_MAX_WORLD);
  *out = nullptr;
  hv_comm* c = new (std::nothrow) hv_comm();
  HV_REQUIRE(c, HV_E_INVALID, "hv_comm_init: out of host memory");
  c->ndev = ndev;
  c->nranks = ndev;
  for (int i = 0; i < ndev; ++i) c->devs[i] = devs[i];
  const ncclResult_t r = ncclCommInitAll(c->comms, ndev, c->devs);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail("ncclCommInitAll", r);
  }
  *out = c;
  return HV_OK;
}

int hv_comm_init_rank(int nranks, int rank, const void* id, int dev, hv_comm** out) {
  HV_REQUIRE(out && id && nranks >= 1 && nranks <= HV_MAX_WORLD && rank >= 0 && rank < nranks,
             HV_E_INVALID, "hv_comm_init_rank: rank %d of %d", rank, nranks);
  *out = nullptr;
  HV_CUDA(cudaSetDevice(dev));
  hv_comm* c = new (std::nothrow) hv_comm();
  HV_REQUIRE(c, HV_E_INVALID, "hv_comm_init_rank: out of host memory");
  c->ndev = 1;
  c->nranks = nranks;
  c->devs[0] = dev;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  const ncclResult_t r = ncclCommInitRank(&c->comms[0], nranks, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail("ncclCommInitRank", r);
  }
  *out = c;
  return HV_OK;
}

int hv_allgather(hv_comm* c, const void* const* send, void* const* recv, size_t bytes,
                 void* const* streams) {
  HV_REQUIRE(c && send && recv && bytes > 0, HV_E_INVALID, "hv_allgather: bad arguments");
  for (int i = 0; i < c->ndev; ++i)
    HV_REQUIRE(send[i] && recv[i], HV_E_INVALID, "hv_allgather: null buffer for device %d",
               c->devs[i]);
  HV_NCCL(ncclGroupStart());
  for (int i = 0; i < c->ndev; ++i) {
    const ncclResult_t r =
        ncclAllGather(send[i], recv[i], bytes, ncclUint8, c->comms[i],
                      streams ? (cudaStream_t)streams[i] : (cudaStream_t)0);
    if (r != ncclSuccess) {
      ncclGroupEnd();
      return nccl_fail("ncclAllGather", r);
    }
  }
  HV_NCCL(ncclGroupEnd());
  return HV_OK;
}

int hv_comm_size(const hv_comm* c, int* nranks, int* ndev) {
  HV_REQUIRE(c && nranks && ndev, HV_E_INVALID, "hv_comm_size: bad arguments");
  *nranks = c->nranks;
  *ndev = c->ndev;
  return HV_OK;
}

int hv_comm_destroy(hv_comm* c) {
  if (!c) return HV_OK;
  int rc = HV_OK;
  for (int i = 0; i < c->ndev; ++i) {
    const ncclResult_t r = ncclCommDestroy(c->comms[i]);
    if (r != ncclSuccess && rc == HV_OK) rc = nccl_fail("ncclCommDestroy", r);
  }
  delete c;
  return rc;
}

}  // extern "C"
