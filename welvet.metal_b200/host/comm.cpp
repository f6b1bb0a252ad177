// NCCL communicator of a head-sharded layer: one all-reduce (sum) of the
// row-sharded output projection per forward / decode step, over NVLink; with
// row-sharded host I/O an all-gather of the input rows and a reduce-scatter of the
// output rows instead.
// The reference is single-device and has no counterpart.
//
// libnccl is opened with dlopen when a communicator is first needed, not linked:
// in a process that already loaded NCCL (e.g. through torch) the same library is
// reused, so two NCCL versions never meet in one process.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "engine.hpp"

namespace wv {
namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclReduceScatter) reduce_scatter = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
  std::string why;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, []() {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.why = std::string("dlopen libnccl.so.2: ") + dlerror();
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.reduce_scatter &&
             api.comm_destroy && api.error_string;
    if (!api.ok) api.why = "libnccl.so.2 lacks an entry point";
  });
  return api;
}

Status nccl_status(ncclResult_t r, const char* what) {
  return Status::err(4, std::string("nccl: ") + what + ": " + nccl().error_string(r));
}

} // namespace

Status comm_unique_id(uint8_t id[128]) {
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  if (!nccl().ok) return Status::err(4, "nccl: " + nccl().why);
  ncclUniqueId u;
  ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return nccl_status(r, "ncclGetUniqueId");
  std::memcpy(id, &u, 128);
  return Status::ok();
}

Status comm_attach(Mha* m, const uint8_t id[128], int nranks, int rank) {
  if (!m || !id || nranks <= 0 || rank < 0 || rank >= nranks) return Status::err(1, "comm: invalid argument");
  if (!nccl().ok) return Status::err(4, "nccl: " + nccl().why);
  comm_release(m);
  WV_CUDA(cudaSetDevice(m->dev->device), "cudaSetDevice");
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  ncclComm_t c = nullptr;
  ncclResult_t r = nccl().comm_init_rank(&c, nranks, u, rank);
  if (r != ncclSuccess) return nccl_status(r, "ncclCommInitRank");
  m->comm = c;
  m->nranks = nranks;
  m->rank = rank;
  WV_CUDA(cudaStreamCreateWithFlags(&m->comm_stream, cudaStreamNonBlocking), "comm stream");
  for (auto& e : m->chunk_done)
    if (!e) WV_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "chunk event");
  WV_CUDA(cudaEventCreateWithFlags(&m->comm_done, cudaEventDisableTiming), "comm event");
  return Status::ok();
}

Status comm_allreduce(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  if (!m->comm || m->nranks == 1) return Status::ok();
  ncclResult_t r = nccl().all_reduce(buf, buf, count, bf16 ? ncclBfloat16 : ncclFloat32, ncclSum,
                                     static_cast<ncclComm_t>(m->comm), s);
  if (r != ncclSuccess) return nccl_status(r, "ncclAllReduce");
  return Status::ok();
}

// In place over buf [nranks * count]: rank r's part starts at r * count elements.
Status comm_allgather(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  if (!m->comm || m->nranks == 1) return Status::ok();
  const size_t es = bf16 ? 2 : 4;
  ncclResult_t r = nccl().all_gather(static_cast<char*>(buf) + (size_t)m->rank * count * es, buf, count,
                                     bf16 ? ncclBfloat16 : ncclFloat32, static_cast<ncclComm_t>(m->comm), s);
  if (r != ncclSuccess) return nccl_status(r, "ncclAllGather");
  return Status::ok();
}
Status comm_reducescatter(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  if (!m->comm || m->nranks == 1) return Status::ok();
  const size_t es = bf16 ? 2 : 4;
  ncclResult_t r = nccl().reduce_scatter(buf, static_cast<char*>(buf) + (size_t)m->rank * count * es, count,
                                         bf16 ? ncclBfloat16 : ncclFloat32, ncclSum,
                                         static_cast<ncclComm_t>(m->comm), s);
  if (r != ncclSuccess) return nccl_status(r, "ncclReduceScatter");
  return Status::ok();
}

void comm_release(Mha* m) {
  if (!m) return;
  if (m->comm) {
    if (nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(m->comm));
    m->comm = nullptr;
    m->nranks = 1;
    m->rank = 0;
  }
  for (auto& e : m->chunk_done) {
    if (e) cudaEventDestroy(e);
    e = nullptr;
  }
  if (m->comm_done) cudaEventDestroy(m->comm_done);
  m->comm_done = nullptr;
  if (m->comm_stream) cudaStreamDestroy(m->comm_stream);
  m->comm_stream = nullptr;
}

} // namespace wv
