// NCCL communicator of a head-sharded layer: one all-reduce (sum) of the
// row-sharded output projection per forward / decode step, over NVLink; with
// row-sharded host I/O an all-gather of the input rows and a reduce-scatter of the
// output rows instead.
// The reference is single-device and has no counterpart.
//
// libnccl is opened with dlopen when a communicator is first needed, not linked:
// in a process that already loaded NCCL (e.g. through torch) the same library is
// reused, so two NCCL versions never meet in one process.
//
// Failures end in a status, never a hang (the reference's contract,
// include/welvet/status.hpp:8-30). The communicator is created non-blocking and
// the host polls ncclCommGetAsyncError until it is ready, for at most the comm
// timeout: a rank that never joins makes every other rank's attach abort the
// communicator (ncclCommAbort) and return code 4. Synchronous calls wait for
// their stream the same way (comm_wait): a collective that does not finish
// within the timeout, or an asynchronous NCCL error, aborts the communicator,
// which ends the NCCL kernels still waiting for a peer, and returns code 4; the
// layer then has no communicator until it is attached again. The timeout is
// WELVET_B200_COMM_TIMEOUT_MS (default 300000 ms), read at each attach.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>
#include <algorithm>

#include "engine.hpp"

namespace wv {
namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) comm_init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclCommAbort) comm_abort = nullptr;
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
    api.comm_init_rank_config =
        reinterpret_cast<decltype(api.comm_init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank_config && api.async_error && api.comm_abort &&
             api.all_reduce && api.all_gather && api.reduce_scatter && api.comm_destroy && api.error_string;
    if (!api.ok) api.why = "libnccl.so.2 lacks an entry point";
  });
  return api;
}

Status nccl_status(ncclResult_t r, const char* what) {
  return Status::err(4, std::string("nccl: ") + what + ": " + nccl().error_string(r));
}

int64_t comm_timeout_ms() {
  const char* v = std::getenv("WELVET_B200_COMM_TIMEOUT_MS");
  if (v && *v) {
    const long long t = std::atoll(v);
    if (t > 0) return t;
  }
  return 300000;
}

// Aborts the layer's communicator after a failure and drops it (the layer runs
// without one until it is attached again). Returns `why`.
Status abort_comm(Mha* m, Status why) {
  if (m->comm && nccl().ok) nccl().comm_abort(static_cast<ncclComm_t>(m->comm));
  m->comm = nullptr;
  m->nranks = 1;
  m->rank = 0;
  return why;
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
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  m->comm_timeout_ms = comm_timeout_ms();
  ncclResult_t r = nccl().comm_init_rank_config(&c, nranks, u, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_status(r, "ncclCommInitRankConfig");
  // Every rank must join within the timeout.
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t state = ncclInProgress;
  while (true) {
    if (nccl().async_error(c, &state) != ncclSuccess) state = ncclInternalError;
    if (state != ncclInProgress) break;
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > m->comm_timeout_ms) {
      nccl().comm_abort(c);
      return Status::err(4, "comm: communicator init timed out after " + std::to_string(m->comm_timeout_ms) +
                                " ms (a rank did not join); aborted");
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (state != ncclSuccess) {
    nccl().comm_abort(c);
    return nccl_status(state, "ncclCommInitRankConfig (asynchronous)");
  }
  m->comm = c;
  m->nranks = nranks;
  m->rank = rank;
  WV_CUDA(cudaStreamCreateWithFlags(&m->comm_stream, cudaStreamNonBlocking), "comm stream");
  for (auto& e : m->chunk_done)
    if (!e) WV_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "chunk event");
  WV_CUDA(cudaEventCreateWithFlags(&m->comm_done, cudaEventDisableTiming), "comm event");
  return Status::ok();
}

namespace {
// A non-blocking communicator may answer an enqueue with ncclInProgress; the
// operation is then complete once the asynchronous state leaves ncclInProgress.
Status enqueued(Mha* m, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return Status::ok();
  if (r != ncclInProgress) return abort_comm(m, nccl_status(r, what));
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t state = ncclInProgress;
  while (true) {
    if (nccl().async_error(static_cast<ncclComm_t>(m->comm), &state) != ncclSuccess) state = ncclInternalError;
    if (state != ncclInProgress) break;
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > m->comm_timeout_ms)
      return abort_comm(m, Status::err(4, std::string("comm: ") + what + " enqueue timed out; communicator aborted"));
    std::this_thread::yield();
  }
  if (state != ncclSuccess) return abort_comm(m, nccl_status(state, what));
  return Status::ok();
}
}  // namespace

Status comm_allreduce(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  if (!m->comm || m->nranks == 1) return Status::ok();
  ncclResult_t r = nccl().all_reduce(buf, buf, count, bf16 ? ncclBfloat16 : ncclFloat32, ncclSum,
                                     static_cast<ncclComm_t>(m->comm), s);
  return enqueued(m, r, "ncclAllReduce");
}

// In place over buf [nranks * count]: rank r's part starts at r * count elements.
Status comm_allgather(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  if (!m->comm || m->nranks == 1) return Status::ok();
  const size_t es = bf16 ? 2 : 4;
  ncclResult_t r = nccl().all_gather(static_cast<char*>(buf) + (size_t)m->rank * count * es, buf, count,
                                     bf16 ? ncclBfloat16 : ncclFloat32, static_cast<ncclComm_t>(m->comm), s);
  return enqueued(m, r, "ncclAllGather");
}
Status comm_reducescatter(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  if (!m->comm || m->nranks == 1) return Status::ok();
  const size_t es = bf16 ? 2 : 4;
  ncclResult_t r = nccl().reduce_scatter(buf, static_cast<char*>(buf) + (size_t)m->rank * count * es, count,
                                         bf16 ? ncclBfloat16 : ncclFloat32, ncclSum,
                                         static_cast<ncclComm_t>(m->comm), s);
  return enqueued(m, r, "ncclReduceScatter");
}

// ------------------------------------------------------- NVLink peer workspace
namespace {
void peer_release(Mha* m) {
  for (int p = 0; p < kPeerMaxRanks; ++p) {
    if (m->peer_areas[p] && m->peer_areas[p] != m->peer_area) cudaIpcCloseMemHandle(m->peer_areas[p]);
    m->peer_areas[p] = nullptr;
  }
  if (m->peer_area) cudaFree(m->peer_area);
  m->peer_area = nullptr;
  m->peer_slot_bytes = m->peer_flags_off = 0;
  m->peer_epoch = 0;
}

bool peer_disabled() {
  static const bool off = [] {
    const char* v = std::getenv("WELVET_B200_PEER_ALLREDUCE");
    return v && v[0] == '0';
  }();
  return off;
}

// All-gathers the CUDA IPC handle of every rank's `own` allocation over NCCL and
// opens the others' (areas[p]; areas[rank] = own). Collective.
Status ipc_exchange(Mha* m, void* own, void** areas, cudaStream_t s) {
  const int n = m->nranks;
  cudaIpcMemHandle_t h;
  WV_CUDA(cudaIpcGetMemHandle(&h, own), "cudaIpcGetMemHandle");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  DevBuf handles;
  WV_TRY(handles.ensure((size_t)n * 64));
  WV_CUDA(cudaMemcpyAsync(static_cast<char*>(handles.p) + (size_t)m->rank * 64, &h, 64, cudaMemcpyHostToDevice, s),
          "peer handle");
  WV_TRY(comm_allgather(m, handles.p, 16, false, s));  // 64 bytes = 16 floats per rank
  WV_TRY(comm_wait(m, s, "peer handle exchange"));
  std::vector<cudaIpcMemHandle_t> all(n);
  WV_CUDA(cudaMemcpy(all.data(), handles.p, (size_t)n * 64, cudaMemcpyDeviceToHost), "peer handles");
  for (int p = 0; p < n; ++p) {
    if (p == m->rank) {
      areas[p] = own;
      continue;
    }
    void* ptr = nullptr;
    WV_CUDA(cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    areas[p] = ptr;
  }
  return Status::ok();
}

// Every rank allocates its receive area (2 parities x n senders x slot bytes, then
// the flags), zeroes it, and the CUDA IPC handles are all-gathered over NCCL; each
// rank opens the others' areas. Collective (same slot size on every rank).
Status peer_setup(Mha* m, size_t bytes, cudaStream_t s) {
  if (m->peer_area && m->peer_slot_bytes >= bytes) return Status::ok();
  peer_release(m);
  const int n = m->nranks;
  const size_t slot = (bytes + 255) / 256 * 256;
  const size_t flags_off = 2 * (size_t)n * slot;
  const size_t total = flags_off + 2 * (size_t)n * kPeerCtas * sizeof(uint32_t);
  WV_CUDA(cudaMalloc(&m->peer_area, total), "peer workspace");
  WV_CUDA(cudaMemsetAsync(m->peer_area, 0, total, s), "peer workspace clear");
  Status st = ipc_exchange(m, m->peer_area, m->peer_areas, s);
  if (!st) {
    peer_release(m);
    return st;
  }
  m->peer_slot_bytes = slot;
  m->peer_flags_off = flags_off;
  m->peer_epoch = 0;
  return Status::ok();
}

void rs_release(Mha* m) {
  for (int p = 0; p < kPeerMaxRanks; ++p) {
    if (m->rs_areas[p] && m->rs_areas[p] != m->rs_area) cudaIpcCloseMemHandle(m->rs_areas[p]);
    m->rs_areas[p] = nullptr;
    if (m->rs_cs[p]) cudaStreamDestroy(m->rs_cs[p]);
    m->rs_cs[p] = nullptr;
    if (m->rs_done[p]) cudaEventDestroy(m->rs_done[p]);
    m->rs_done[p] = nullptr;
  }
  if (m->rs_area) cudaFree(m->rs_area);
  m->rs_area = nullptr;
  if (m->rs_epoch_tab) cudaFree(m->rs_epoch_tab);
  m->rs_epoch_tab = nullptr;
  m->rs_slice_bytes = m->rs_flags_off = 0;
  m->rs_chunks = 0;
  m->rs_epoch = m->rs_calls = 0;
}

constexpr uint32_t kEpochs = 4096;  // flag values 1 .. kEpochs - 1, reused cyclically

// Collective (the same chunks and slice size on every rank).
Status rs_setup(Mha* m, int chunks, size_t slice_bytes, cudaStream_t s) {
  if (m->rs_area && m->rs_chunks >= chunks && m->rs_slice_bytes >= slice_bytes) return Status::ok();
  rs_release(m);
  const int n = m->nranks;
  const size_t slice = (slice_bytes + 255) / 256 * 256;
  const size_t flags_off = 2 * (size_t)chunks * n * slice;
  const size_t total = flags_off + 2 * (size_t)chunks * n * sizeof(uint32_t);
  WV_CUDA(cudaMalloc(&m->rs_area, total), "reduce-scatter workspace");
  WV_CUDA(cudaMemsetAsync(static_cast<char*>(m->rs_area) + flags_off, 0, total - flags_off, s), "flags clear");
  std::vector<uint32_t> tab(kEpochs);
  for (uint32_t i = 0; i < kEpochs; ++i) tab[i] = i;
  WV_CUDA(cudaMalloc(&m->rs_epoch_tab, kEpochs * sizeof(uint32_t)), "epoch table");
  WV_CUDA(cudaMemcpyAsync(m->rs_epoch_tab, tab.data(), kEpochs * sizeof(uint32_t), cudaMemcpyHostToDevice, s),
          "epoch table");
  Status st = ipc_exchange(m, m->rs_area, m->rs_areas, s);  // (its comm_wait also completes the copy above)
  if (!st) {
    rs_release(m);
    return st;
  }
  for (int p = 0; p < n; ++p) {
    if (p == m->rank) continue;
    WV_CUDA(cudaStreamCreateWithFlags(&m->rs_cs[p], cudaStreamNonBlocking), "copy stream");
    WV_CUDA(cudaEventCreateWithFlags(&m->rs_done[p], cudaEventDisableTiming), "copy event");
  }
  m->rs_slice_bytes = slice;
  m->rs_flags_off = flags_off;
  m->rs_chunks = chunks;
  return Status::ok();
}

bool rs_disabled() {
  static const bool off = [] {
    const char* v = std::getenv("WELVET_B200_PEER_RS");
    return v && v[0] == '0';
  }();
  return off;
}
}  // namespace

bool comm_peer_rs_ok(const Mha* m) {
  return m->comm && m->nranks > 1 && m->nranks <= kPeerMaxRanks && !rs_disabled();
}

Status comm_peer_rs_chunk(Mha* m, char* base, int64_t rows, int64_t max_rows, int dm, bool bf16, int chunk,
                          int chunks, cudaEvent_t ready, cudaStream_t st) {
  const int n = m->nranks;
  const size_t es = bf16 ? 2 : 4;
  if (!comm_peer_rs_ok(m) || rows % n || max_rows % n || chunk < 0 || chunk >= chunks)
    return Status::err(2, "comm: peer reduce-scatter not available here");
  const size_t slice = (size_t)(rows / n) * dm * es;
  if (slice % 16) return Status::err(2, "comm: peer reduce-scatter needs 16-byte slices");
  WV_TRY(rs_setup(m, chunks, (size_t)(max_rows / n) * dm * es, st));
  if (chunk == 0) ++m->rs_calls;
  const size_t cp = m->rs_calls & 1;
  const uint32_t epoch = m->rs_epoch++ % (kEpochs - 1) + 1;
  const size_t slot0 = (cp * m->rs_chunks + chunk) * n;  // first slot of this (call parity, chunk)
  for (int p = 0; p < n; ++p) {
    if (p == m->rank) continue;
    char* area = static_cast<char*>(m->rs_areas[p]);
    WV_CUDA(cudaStreamWaitEvent(m->rs_cs[p], ready, 0), "wait");
    WV_CUDA(cudaMemcpyAsync(area + (slot0 + m->rank) * m->rs_slice_bytes, base + (size_t)p * slice, slice,
                            cudaMemcpyDeviceToDevice, m->rs_cs[p]),
            "slice to peer");
    // issued after the slice on the same stream: written once the slice has landed
    WV_CUDA(cudaMemcpyAsync(area + m->rs_flags_off + (slot0 + m->rank) * sizeof(uint32_t), m->rs_epoch_tab + epoch,
                            sizeof(uint32_t), cudaMemcpyDeviceToDevice, m->rs_cs[p]),
            "flag to peer");
  }
  PeerRsArgs a;
  a.own = base + (size_t)m->rank * slice;
  a.slots = static_cast<char*>(m->rs_area) + slot0 * m->rs_slice_bytes;
  a.flags = reinterpret_cast<const uint32_t*>(static_cast<char*>(m->rs_area) + m->rs_flags_off) + slot0;
  a.count = (size_t)(rows / n) * dm;
  a.slot_bytes = m->rs_slice_bytes;
  a.bf16 = bf16 ? 1 : 0;
  a.nranks = n;
  a.rank = m->rank;
  a.epoch = epoch;
  a.wait_ns = (uint64_t)std::min<int64_t>(m->comm_timeout_ms, 60000) * 1000000ull;
  a.err = m->dev->err;
  WV_CUDA(peer_rs_sum(a, 2 * m->dev->sm_count, st), "peer_rs_sum");
  count_launch();
  return Status::ok();
}

Status comm_peer_rs_finish(Mha* m, cudaStream_t s) {
  for (int p = 0; p < m->nranks; ++p) {
    if (p == m->rank || !m->rs_cs[p]) continue;
    WV_CUDA(cudaEventRecord(m->rs_done[p], m->rs_cs[p]), "event");
    WV_CUDA(cudaStreamWaitEvent(s, m->rs_done[p], 0), "wait");
  }
  return Status::ok();
}

// ------------------------------------------ attention-output exchange (mode 2)
namespace {
void xa_release(Mha* m) {
  for (int p = 0; p < kPeerMaxRanks; ++p) {
    if (m->xa_areas[p] && m->xa_areas[p] != m->xa_area) cudaIpcCloseMemHandle(m->xa_areas[p]);
    m->xa_areas[p] = nullptr;
    if (m->xa_cs[p]) cudaStreamDestroy(m->xa_cs[p]);
    m->xa_cs[p] = nullptr;
    if (m->xa_done[p]) cudaEventDestroy(m->xa_done[p]);
    m->xa_done[p] = nullptr;
  }
  if (m->xa_area) cudaFree(m->xa_area);
  m->xa_area = nullptr;
  if (m->xa_epoch_tab) cudaFree(m->xa_epoch_tab);
  m->xa_epoch_tab = nullptr;
  m->xa_slot_bytes = m->xa_flags_off = 0;
  m->xa_chunks = 0;
  m->xa_epoch = m->xa_calls = 0;
  m->wo_full.release();
}

// Collective (the same chunks and slot size on every rank): receive area, flags,
// IPC mappings, copy streams and the gathered Wo.
Status xa_setup(Mha* m, int chunks, size_t slot_bytes, cudaStream_t s) {
  if (m->xa_area && m->xa_chunks >= chunks && m->xa_slot_bytes >= slot_bytes) return Status::ok();
  xa_release(m);
  const int n = m->nranks;
  const size_t slot = (slot_bytes + 255) / 256 * 256;
  const size_t flags_off = 2 * (size_t)chunks * slot;
  const size_t total = flags_off + 2 * (size_t)chunks * n * sizeof(uint32_t);
  WV_CUDA(cudaMalloc(&m->xa_area, total), "exchange workspace");
  WV_CUDA(cudaMemsetAsync(static_cast<char*>(m->xa_area) + flags_off, 0, total - flags_off, s), "flags clear");
  std::vector<uint32_t> tab(kEpochs);
  for (uint32_t i = 0; i < kEpochs; ++i) tab[i] = i;
  WV_CUDA(cudaMalloc(&m->xa_epoch_tab, kEpochs * sizeof(uint32_t)), "epoch table");
  WV_CUDA(cudaMemcpyAsync(m->xa_epoch_tab, tab.data(), kEpochs * sizeof(uint32_t), cudaMemcpyHostToDevice, s),
          "epoch table");
  Status st = ipc_exchange(m, m->xa_area, m->xa_areas, s);
  if (!st) {
    xa_release(m);
    return st;
  }
  for (int p = 0; p < n; ++p) {
    if (p == m->rank) continue;
    WV_CUDA(cudaStreamCreateWithFlags(&m->xa_cs[p], cudaStreamNonBlocking), "copy stream");
    WV_CUDA(cudaEventCreateWithFlags(&m->xa_done[p], cudaEventDisableTiming), "copy event");
  }
  // Every head's Wo columns: the ranks' [d, q_dim_l] shards are all-gathered (rank
  // blocks one after another) and laid out as [d, q_dim], rank p's block in columns
  // [p q_dim_l, (p+1) q_dim_l) (the exchange's column order).
  const int64_t dm = m->cfg.c.d_model, qdl = m->qd_l;
  DevBuf gathered;
  WV_TRY(gathered.ensure((size_t)n * dm * qdl * 2));
  WV_CUDA(cudaMemcpyAsync(gathered.as<char>() + (size_t)m->rank * dm * qdl * 2, m->wo.p, (size_t)dm * qdl * 2,
                          cudaMemcpyDeviceToDevice, s), "Wo shard");
  WV_TRY(comm_allgather(m, gathered.p, (size_t)dm * qdl, true, s));
  WV_TRY(m->wo_full.ensure((size_t)dm * qdl * n * 2));
  for (int p = 0; p < n; ++p)
    WV_CUDA(cudaMemcpy2DAsync(m->wo_full.as<char>() + (size_t)p * qdl * 2, (size_t)n * qdl * 2,
                              gathered.as<char>() + (size_t)p * dm * qdl * 2, (size_t)qdl * 2, (size_t)qdl * 2, dm,
                              cudaMemcpyDeviceToDevice, s), "Wo layout");
  WV_TRY(comm_wait(m, s, "exchange set-up"));  // `gathered` is freed on return
  m->xa_slot_bytes = slot;
  m->xa_flags_off = flags_off;
  m->xa_chunks = chunks;
  return Status::ok();
}

bool xa_disabled() {
  static const bool off = [] {
    const char* v = std::getenv("WELVET_B200_PEER_XA");
    return v && v[0] == '0';
  }();
  return off;
}
}  // namespace

bool comm_xa_ok(const Mha* m) {
  return m->comm && m->nranks > 1 && m->nranks <= kPeerMaxRanks && m->precision == 1 && m->wfmt == 0 &&
         m->qd_l * m->nranks == m->cfg.qd && ((int64_t)m->qd_l * 2) % 16 == 0 && !xa_disabled();
}

Status comm_xa_chunk(Mha* m, const char* attn, int64_t rows, int64_t max_rows, int chunk, int chunks,
                     cudaEvent_t ready, cudaStream_t s, const void** a_out) {
  const int n = m->nranks;
  if (!comm_xa_ok(m) || rows % n || max_rows % n || chunk < 0 || chunk >= chunks || chunks > Mha::kMaxChunks)
    return Status::err(2, "comm: attention-output exchange not available here");
  const int64_t own = rows / n, qdl = m->qd_l, qd = (int64_t)qdl * n;
  WV_TRY(xa_setup(m, chunks, (size_t)(max_rows / n) * qd * 2, s));
  if (chunk == 0) ++m->xa_calls;
  const size_t cp = m->xa_calls & 1;
  const uint32_t epoch = m->xa_epoch++ % (kEpochs - 1) + 1;
  m->xa_chunk_epoch[chunk] = epoch;
  const size_t slot = cp * m->xa_chunks + chunk;  // (call parity, chunk)
  const size_t flag0 = slot * n;                  // its first flag
  // rows [p own, (p+1) own) of this chunk go to rank p, into columns [rank qdl, ...)
  for (int p = 0; p < n; ++p) {
    char* dst = static_cast<char*>(m->xa_areas[p]) + slot * m->xa_slot_bytes + (size_t)m->rank * qdl * 2;
    const char* src = attn + (size_t)p * own * qdl * 2;
    if (p == m->rank) {
      WV_CUDA(cudaMemcpy2DAsync(dst, (size_t)qd * 2, src, (size_t)qdl * 2, (size_t)qdl * 2, own,
                                cudaMemcpyDeviceToDevice, s), "own block");
      continue;
    }
    WV_CUDA(cudaStreamWaitEvent(m->xa_cs[p], ready, 0), "wait");
    WV_CUDA(cudaMemcpy2DAsync(dst, (size_t)qd * 2, src, (size_t)qdl * 2, (size_t)qdl * 2, own,
                              cudaMemcpyDeviceToDevice, m->xa_cs[p]), "block to peer");
    // issued after the block on the same stream: written once the block has landed
    WV_CUDA(cudaMemcpyAsync(static_cast<char*>(m->xa_areas[p]) + m->xa_flags_off + (flag0 + m->rank) * 4,
                            m->xa_epoch_tab + epoch, 4, cudaMemcpyDeviceToDevice, m->xa_cs[p]),
            "flag to peer");
  }
  *a_out = static_cast<const char*>(m->xa_area) + slot * m->xa_slot_bytes;
  return Status::ok();
}

Status comm_xa_wait(Mha* m, int chunk, cudaStream_t s) {
  if (!m->xa_area || chunk < 0 || chunk >= m->xa_chunks) return Status::err(4, "comm: exchange not set up");
  const size_t slot = (m->xa_calls & 1) * m->xa_chunks + chunk;
  const uint32_t* flags =
      reinterpret_cast<const uint32_t*>(static_cast<const char*>(m->xa_area) + m->xa_flags_off) + slot * m->nranks;
  const uint64_t wait_ns = (uint64_t)std::min<int64_t>(m->comm_timeout_ms, 60000) * 1000000ull;
  WV_CUDA(peer_flags_wait(flags, m->nranks, m->rank, m->xa_chunk_epoch[chunk], wait_ns, m->dev->err, s),
          "peer_flags_wait");
  count_launch();
  return Status::ok();
}

Status comm_xa_finish(Mha* m, cudaStream_t s) {
  for (int p = 0; p < m->nranks; ++p) {
    if (p == m->rank || !m->xa_cs[p]) continue;
    WV_CUDA(cudaEventRecord(m->xa_done[p], m->xa_cs[p]), "event");
    WV_CUDA(cudaStreamWaitEvent(s, m->xa_done[p], 0), "wait");
  }
  return Status::ok();
}

bool comm_peer_ok(const Mha* m, size_t bytes) {
  return m->comm && m->nranks > 1 && m->nranks <= kPeerMaxRanks && bytes > 0 && bytes % 16 == 0 &&
         bytes <= kPeerMaxBytes && !peer_disabled();
}

Status comm_peer_allreduce(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s) {
  const size_t bytes = count * (bf16 ? 2 : 4);
  if (!comm_peer_ok(m, bytes)) return Status::err(2, "comm: peer all-reduce not available here");
  WV_TRY(peer_setup(m, bytes, s));
  PeerArgs a;
  a.in = buf;
  a.out = buf;
  a.count = count;
  a.bf16 = bf16 ? 1 : 0;
  a.nranks = m->nranks;
  a.rank = m->rank;
  for (int p = 0; p < m->nranks; ++p) a.areas[p] = m->peer_areas[p];
  a.slot_bytes = m->peer_slot_bytes;
  a.flags_off = m->peer_flags_off;
  a.epoch = ++m->peer_epoch;
  // The device wait is bounded like the host's collective waits (capped at 60 s).
  a.wait_ns = (uint64_t)std::min<int64_t>(m->comm_timeout_ms, 60000) * 1000000ull;
  a.err = m->dev->err;
  WV_CUDA(peer_allreduce(a, s), "peer_allreduce");
  count_launch();
  return Status::ok();
}

Status comm_poll(Mha* m) {
  if (!m->comm || !nccl().ok) return Status::ok();
  ncclResult_t state = ncclSuccess;
  ncclResult_t r = nccl().async_error(static_cast<ncclComm_t>(m->comm), &state);
  if (r != ncclSuccess) return abort_comm(m, nccl_status(r, "ncclCommGetAsyncError"));
  if (state != ncclSuccess && state != ncclInProgress)
    return abort_comm(m, nccl_status(state, "asynchronous communicator error; communicator aborted"));
  return Status::ok();
}

Status comm_wait(Mha* m, cudaStream_t s, const char* what) {
  if (!m->comm || m->nranks == 1) {
    WV_CUDA(cudaStreamSynchronize(s), what);
    return Status::ok();
  }
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return comm_poll(m);
    if (e != cudaErrorNotReady) return cuda_status(e, what);
    WV_TRY(comm_poll(m));
    if (!m->comm) return Status::err(4, "comm: communicator aborted");
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > m->comm_timeout_ms) {
      Status st = abort_comm(m, Status::err(4, std::string("comm: ") + what + " did not finish within " +
                                                   std::to_string(m->comm_timeout_ms) +
                                                   " ms (a peer rank stopped); communicator aborted"));
      // the abort ends the NCCL kernels that waited for the peer; drain the stream
      cudaStreamSynchronize(s);
      cudaGetLastError();
      return st;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

void comm_release(Mha* m) {
  if (!m) return;
  peer_release(m);
  rs_release(m);
  xa_release(m);
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
