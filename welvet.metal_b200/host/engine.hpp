// Host orchestration of the B200 MHA path (the role of the reference's
// src/layers/mha/mha.cpp + src/layers/dense/dense.cpp + src/metal/*.mm):
// configuration checks with the reference's defaults, resident weights in HBM,
// the forward / prefill / decode sequences of kernel launches, the paged KV
// cache and the NCCL communicator of a head shard.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/welvet_b200.h"
#include "../csrc/kernels.h"

namespace wv {

struct Status {
  int code = 0;  // welvet_status codes
  std::string msg;
  static Status ok() { return {}; }
  static Status err(int c, std::string m) { return {c, std::move(m)}; }
  explicit operator bool() const { return code == 0; }
};

welvet_status to_c(const Status& s);
Status cuda_status(cudaError_t e, const char* what);

// Keeps the calling thread's current CUDA device across an entry point: the
// engine switches to the device of the layer it runs, and the destructor
// switches back. When the caller's device has no active primary context (the
// thread never used CUDA on it), switching back would create one on that device
// (cudaSetDevice initialises it), so the thread is then left on the device the
// call used.
class DeviceRestore {
 public:
  DeviceRestore();
  ~DeviceRestore();
  DeviceRestore(const DeviceRestore&) = delete;
  DeviceRestore& operator=(const DeviceRestore&) = delete;

 private:
  int dev_ = -1;
};

#define WV_TRY(expr)                               \
  do {                                             \
    ::wv::Status _st = (expr);                     \
    if (!_st) return _st;                          \
  } while (0)
#define WV_CUDA(expr, what)                                    \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return ::wv::cuda_status(_e, what); \
  } while (0)

// Kernel launches issued by this library (benchmark accounting).
extern std::atomic<int64_t> g_launches;
inline void count_launch(int n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// Live per-kernel timing: when enabled, the engine brackets each hot kernel with
// CUDA events on the stream it launches on; profile_read() synchronises and
// accumulates the durations per kernel id.
enum ProfId : int {
  kProfGemmQkv = 0,
  kProfAttnPrefill = 1,
  kProfGemmO = 2,
  kProfAttnDecode = 3,
  kProfGemmQkvDecode = 4,
  kProfGemmODecode = 5,
  kProfAllReduce = 6,
  kProfOther = 7,
  kProfGemmGateUp = 8,   // SwiGLU Gate|Up GEMM with the SiLU * up epilogue
  kProfGemmDown = 9,     // SwiGLU Down GEMM
  kProfNorm = 10,        // RMSNorm / LayerNorm
  kProfEmbedding = 11,
  kProfAttnBwd = 12,     // NormalBP attention backward
  kProfGemmGrad = 13,    // NormalBP gradient GEMMs
  kProfCount = 14,
};
void prof_enable(bool on);
bool prof_on();
void prof_begin(int id, cudaStream_t s);
void prof_end(int id, cudaStream_t s);
void prof_read(double* ms, int64_t* counts, bool reset);

// Owned device allocation, grown on demand (never shrunk).
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  Status ensure(size_t n) {
    if (n <= bytes && p) return Status::ok();
    release();
    cudaError_t e = cudaMalloc(&p, n ? n : 16);
    if (e != cudaSuccess) {
      p = nullptr;
      return cuda_status(e, "cudaMalloc");
    }
    bytes = n;
    return Status::ok();
  }
  template <class T> T* as() const { return static_cast<T*>(p); }
};

// Per-device state shared by every layer on that device.
struct DeviceCtx {
  int device = 0;
  int sm_count = 148;
  int cc_major = 0, cc_minor = 0;
  std::string name;
  uint32_t* err = nullptr;     // device error word
  float* scratch = nullptr;    // 4096 floats (reductions)
  float* scalars = nullptr;    // 64 floats (per-tensor scales)
  int* tile_ctr = nullptr;     // tile counter of the standalone persistent attention entry
};
Status device_ctx(int device, DeviceCtx** out);  // device < 0: current
Status check_device_error(DeviceCtx* d);         // sync + read/clear the error word
// Reads and clears the error word of welvet_b200_decode_attention_static on the
// current device (decode_static.cu; 0 when that entry point has not run there).
Status take_static_decode_error(uint32_t* code);

// Resolved welvet::mha::Config (defaults of validate(),
// src/layers/mha/mha.cpp:63-94) + execution choices.
struct Cfg {
  welvet_b200_mha_config c{};
  int hd = 0, nk = 0, msl = 0, group = 0;
  int qd = 0, kd = 0;
  float scale = 0.f;
  bool rope = false, alibi = false;
};
Status resolve_config(const welvet_b200_mha_config& in, Cfg* out);

struct Kv;

struct Mha {
  Cfg cfg;
  DeviceCtx* dev = nullptr;
  int h0 = 0, hc = 0, kh0 = 0, khc = 0;  // head shard
  int qd_l = 0, kd_l = 0, nqkv = 0;
  int precision = 0, wfmt = 0;
  int wdtype = 1;  // FormatNone dtype of resident codes (weight_format 3)
  // weights (layouts documented in engine.cpp)
  DevBuf wqkv, wqkv_lo, wo, wo_lo, wqkv_scale, wo_scale;
  // RoPE cos/sin table
  DevBuf rope_tab;
  int rope_max_pos = 0;
  // workspaces
  DevBuf x_io, pre_io, post_io, x_hi, x_lo, qkv, attn, attn_hi, attn_lo, post_tmp;
  DevBuf positions, slots;
  DevBuf splitk_ws;  // split-K partial sums of the decode projections
  DevBuf qkv_hi, qkv_lo;  // FP32 path: TF32 split of q/k/v for the 3xTF32 attention
  DevBuf attn_ctr;        // tile counter of the persistent prefill attention (one int)
  // communicator (head-sharded tensor parallelism); the all-reduce of a forward
  // chunk runs on comm_stream while the next chunk computes on the caller's stream
  void* comm = nullptr;
  int nranks = 1, rank = 0;
  int64_t comm_timeout_ms = 300000;  // bound of init, enqueue and synchronous waits
  // Output collective of a device-buffer forward with a communicator: 0 all-reduce
  // (every rank holds every summed row), 1 reduce-scatter (see welvet_b200.h).
  int out_mode = 0;
  cudaStream_t comm_stream = nullptr;
  // NVLink peer workspace of the peer-memory all-reduce (decode outputs): this
  // rank's receive area and every rank's area opened through CUDA IPC (index =
  // rank). Created collectively by the first call that needs it (comm.cpp).
  void* peer_area = nullptr;
  void* peer_areas[8] = {};
  size_t peer_slot_bytes = 0, peer_flags_off = 0;
  uint32_t peer_epoch = 0;
  // Copy-engine reduce-scatter of the chunked prefill output (device buffers, output
  // mode 1): receive area [2 call parities][chunks][N senders][slice] then flags
  // [2][chunks][N], every rank's area opened through CUDA IPC, one copy stream per
  // peer, and a device table of epoch values for the flag writes.
  void* rs_area = nullptr;
  void* rs_areas[8] = {};
  size_t rs_slice_bytes = 0, rs_flags_off = 0;
  int rs_chunks = 0;
  cudaStream_t rs_cs[8] = {};
  cudaEvent_t rs_done[8] = {};
  uint32_t* rs_epoch_tab = nullptr;
  uint32_t rs_epoch = 0, rs_calls = 0;
  // Attention-output exchange of the chunked prefill (device buffers, output mode 2):
  // receive area [2 call parities][chunks][rows/N x q_dim] (the output projection's
  // A operand: sender p's heads in columns [p q_dim_l, (p+1) q_dim_l)), then flags
  // [2][chunks][N]; every rank's area opened through CUDA IPC, one copy stream per
  // peer, a device table of epoch values for the flag writes, and every head's Wo
  // columns [d, q_dim] gathered from the ranks on first use.
  void* xa_area = nullptr;
  void* xa_areas[8] = {};
  size_t xa_slot_bytes = 0, xa_flags_off = 0;
  int xa_chunks = 0;
  cudaStream_t xa_cs[8] = {};
  cudaEvent_t xa_done[8] = {};
  uint32_t* xa_epoch_tab = nullptr;
  uint32_t xa_epoch = 0, xa_calls = 0;
  uint32_t xa_chunk_epoch[16] = {};
  DevBuf wo_full;
  static constexpr int kMaxChunks = 16;
  cudaEvent_t chunk_done[kMaxChunks] = {};
  cudaEvent_t comm_done = nullptr;
  // host-buffer calls: input copies (io_in) and output copies (io_out) of the chunks
  cudaStream_t io_in = nullptr, io_out = nullptr;
  cudaEvent_t io_ev[2 * kMaxChunks + 1] = {};
  cudaEvent_t gather_ev[kMaxChunks] = {};  // row-sharded host I/O: chunk all-gathered
  std::mutex mu;  // one call at a time per layer (reference: per-session lock)
  ~Mha();
};

Status mha_mount(const welvet_b200_mha_config& cfg, int dtype, const float* Q, const float* K,
                 const float* V, const float* O, bool on_device, Mha** out);
// Replaces the weights of an FP32 full-head layer by decoded device matrices
// (W_qkv rows Q | K | V, Wo), without allocating.
Status mha_reload_fp32(Mha* m, const float* wqkv, const float* wo, cudaStream_t s);
Status mha_forward(Mha* m, int batch, int seq, const void* x, void* pre, void* post,
                   bool on_device, cudaStream_t s, Kv* kv = nullptr, bool rows = false);
// rows = true (host buffers, communicator of N ranks, per-sequence mode, no pre):
// batch is the whole batch, x / post hold this rank's batch / N sequences
// (ranks in order); the input rows are all-gathered and the output rows
// reduce-scattered over NVLink, so each GPU copies 1/N of them over PCIe.

struct Kv {
  Mha* layer = nullptr;
  int max_batch = 0, max_ctx = 0, pages_per_seq = 0;
  DevBuf k_pool, v_pool, block_table, ctx_len, scratch;
  std::vector<int> ctx_host;
};
Status kv_create(Mha* m, int max_batch, int max_ctx, Kv** out);
Status kv_fill(Kv* kv, int batch, int ctx, const void* k, const void* v, bool on_device,
               cudaStream_t s);
Status mha_decode(Mha* m, Kv* kv, int batch, const void* x, void* pre, void* post,
                  bool on_device, cudaStream_t s);

// NCCL (comm.cpp)
Status comm_unique_id(uint8_t id[128]);
Status comm_attach(Mha* m, const uint8_t id[128], int nranks, int rank);
Status comm_allreduce(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s);
// in place over buf [nranks * count]; rank r's part at r * count elements
Status comm_allgather(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s);
Status comm_reducescatter(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s);
// All-reduce of a small vector through the NVLink peer workspace (one kernel, no
// NCCL): true when this layer can take it (2-8 ranks, at most kPeerMaxBytes, 16-byte
// multiple, not switched off by WELVET_B200_PEER_ALLREDUCE=0). Collective: every
// rank makes the same calls; the first one (and any larger one) sets the workspace up.
constexpr size_t kPeerMaxBytes = 4u << 20;
bool comm_peer_ok(const Mha* m, size_t bytes);
Status comm_peer_allreduce(Mha* m, void* buf, size_t count, bool bf16, cudaStream_t s);
// Reduce-scatter of one chunk of a device-buffer forward's output through copy
// engines and peer memory (no NCCL kernels on the SMs): the chunk's rows [base,
// base + rows) (rows divisible by the ranks; the first chunk of a call has chunk 0)
// are sent slice by slice to their owners once `ready` (recorded on the compute
// stream after the chunk's output projection) has passed, and this rank's slice is
// summed in place by a kernel on st. Collective, like NCCL; true from comm_peer_rs_ok
// when the layer can take it (2-8 ranks; WELVET_B200_PEER_RS=0 keeps NCCL).
bool comm_peer_rs_ok(const Mha* m);
Status comm_peer_rs_chunk(Mha* m, char* base, int64_t rows, int64_t max_rows, int dm, bool bf16, int chunk,
                          int chunks, cudaEvent_t ready, cudaStream_t st);
// s waits until every copy of the call has read the output rows.
Status comm_peer_rs_finish(Mha* m, cudaStream_t s);
// Attention-output exchange of one chunk of a device-buffer forward (output mode 2,
// BF16 layers with format-0 weights, 2-8 ranks; WELVET_B200_PEER_XA=0 turns it
// off): once `ready` (recorded on s after the chunk's attention) has passed, rows
// [p rows/N, (p+1) rows/N) of this rank's attention output `attn` [rows, q_dim_l]
// go by copy engine into rank p's receive slot, columns [rank q_dim_l, ...), and
// this rank's own block by a copy on s. *a_out = this rank's slot [rows/N, q_dim],
// complete once comm_xa_wait(chunk) has passed on s. The first call sets up the
// receive areas and gathers every head's Wo (m->wo_full). Collective.
bool comm_xa_ok(const Mha* m);
Status comm_xa_chunk(Mha* m, const char* attn, int64_t rows, int64_t max_rows, int chunk, int chunks,
                     cudaEvent_t ready, cudaStream_t s, const void** a_out);
Status comm_xa_wait(Mha* m, int chunk, cudaStream_t s);
// s waits until every copy of the call has read the attention rows.
Status comm_xa_finish(Mha* m, cudaStream_t s);
// Asynchronous NCCL error check; on an error the communicator is aborted and
// dropped, code 4.
Status comm_poll(Mha* m);
// cudaStreamSynchronize for synchronous calls of a layer with a communicator:
// polls the stream and the communicator, aborts the communicator after
// comm_timeout_ms, code 4 on either failure.
Status comm_wait(Mha* m, cudaStream_t s, const char* what);
void comm_release(Mha* m);

// small device helpers (engine_kernels.cu)
cudaError_t make_prefill_slots(int* slots, int batch, int seq, int pages_per_seq, cudaStream_t s);
cudaError_t make_decode_rows(int* ctx, int* positions, int* slots, int batch, int pages_per_seq,
                             cudaStream_t s);
cudaError_t set_ctx(int* ctx, int batch, int value, cudaStream_t s);
cudaError_t make_block_table(int* bt, int batch, int pages_per_seq, cudaStream_t s);

} // namespace wv
