// NCCL communicator of a head-sharded layer: one all-reduce (sum) of the
// row-sharded output projection per forward / decode step, over NVLink.
// The reference is single-device and has no counterpart.
#include <nccl.h>

#include <cstring>

#include "engine.hpp"

namespace wv {

static Status nccl_status(ncclResult_t r, const char* what) {
  return Status::err(4, std::string("nccl: ") + what + ": " + ncclGetErrorString(r));
}

Status comm_unique_id(uint8_t id[128]) {
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  ncclUniqueId u;
  ncclResult_t r = ncclGetUniqueId(&u);
  if (r != ncclSuccess) return nccl_status(r, "ncclGetUniqueId");
  std::memcpy(id, &u, 128);
  return Status::ok();
}

Status comm_attach(Mha* m, const uint8_t id[128], int nranks, int rank) {
  if (!m || !id || nranks <= 0 || rank < 0 || rank >= nranks) return Status::err(1, "comm: invalid argument");
  comm_release(m);
  WV_CUDA(cudaSetDevice(m->dev->device), "cudaSetDevice");
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  ncclComm_t c = nullptr;
  ncclResult_t r = ncclCommInitRank(&c, nranks, u, rank);
  if (r != ncclSuccess) return nccl_status(r, "ncclCommInitRank");
  m->comm = c;
  m->nranks = nranks;
  m->rank = rank;
  return Status::ok();
}

Status comm_allreduce(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  if (!m->comm || m->nranks == 1) return Status::ok();
  ncclResult_t r = ncclAllReduce(buf, buf, count, bf16 ? ncclBfloat16 : ncclFloat32, ncclSum,
                                 static_cast<ncclComm_t>(m->comm), s);
  if (r != ncclSuccess) return nccl_status(r, "ncclAllReduce");
  return Status::ok();
}

void comm_release(Mha* m) {
  if (m && m->comm) {
    ncclCommDestroy(static_cast<ncclComm_t>(m->comm));
    m->comm = nullptr;
    m->nranks = 1;
    m->rank = 0;
  }
}

} // namespace wv
