// Split-KV decode attention that allocates nothing.
//
// The layer-level decode (mha_decode) keeps its split partials in a buffer of
// the KV cache that grows on demand with cudaMalloc. Some callers cannot let a
// library allocate device memory while they decode:
//   * a serving loop whose HBM is reserved up front by its own pool allocator
//     (the KV pages, the activations and the weights fill the device), so a
//     late cudaMalloc can fail, and cudaFree synchronises the whole device,
//     stalling the other streams of the loop;
//   * a host framework that owns all device memory through its own caching
//     allocator (PyTorch's, for one) and sizes its pools against the free
//     memory it sees: memory that a library takes behind its back is missing
//     from that accounting and can make the framework's next allocation fail.
// For them this entry point runs the same kernels as the layer's decode step
// (attn_decode: decode_tc_kernel for BF16 head_dim 64/128 with aligned rows, else
// the CUDA-core decode_kernel, then decode_combine_kernel) with the partials in a
// fixed file-scope device array.
//
// Contract:
//   * The scratch holds kStaticDecodeFloats floats (4 MiB) per device. A call
//     needs batch * heads * splits * (head_dim + 2) floats; the split count is
//     lowered until it fits, and a call that does not fit even with one split is
//     rejected with code 1 before anything is launched.
//   * Nothing has to start at zero: every split block writes all head_dim + 2
//     values (o, m, l) of its slot before the combine kernel reads them, also
//     when its key range is empty (m = -inf, l = 0, o = 0).
//   * One scratch per device is shared by every call on that device: calls that
//     overlap in time (different streams, or different host threads with their
//     own streams) race on it. Issue them on one stream, one after another.
//   * Errors found on the device (a bounded wait of decode_tc_kernel that ran
//     out) go to a second file-scope word, g_decode_err, found the same way, so
//     that no error buffer has to be allocated either. welvet_b200_device_check
//     reads and clears it together with the library's per-device error word
//     (that call allocates the library's small per-device state on its first
//     call on a device, so callers that cannot allocate later make it once
//     during their set-up).
//   * Page ids in block_table must name pages of k_pool/v_pool: the entry point
//     does not know the pools' size, so it cannot check them.
//   * The caller's current device is restored before the call returns.
//   * The first call on a device performs the set-up: the symbol lookup below
//     (which can load this module and its 4 MiB array) and the first launches of
//     the decode kernels (which load their module). Make that first call before
//     any stream capture begins.
#include <cuda_runtime.h>

#include <mutex>

#include "engine.hpp"

namespace wv {
namespace {

constexpr size_t kStaticDecodeFloats = WELVET_B200_DECODE_STATIC_FLOATS;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_decode_partial[kStaticDecodeFloats];
static __device__ uint32_t g_decode_err;

struct StaticSlot {
  float* partial = nullptr;
  uint32_t* err = nullptr;
  int sm_count = 0;
};
StaticSlot g_slots[kMaxDevices];
std::mutex g_slots_mu;

// Once per device, with that device current: address of this module's copy of
// g_decode_partial, and the SM count used to size the splits.
Status static_slot(int device, StaticSlot* out) {
  std::lock_guard<std::mutex> lock(g_slots_mu);
  StaticSlot& s = g_slots[device];
  if (!s.partial) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_partial);
    if (e != cudaSuccess) return cuda_status(e, "decode_attention_static: cudaGetSymbolAddress");
    void* pe = nullptr;
    e = cudaGetSymbolAddress(&pe, g_decode_err);
    if (e != cudaSuccess) return cuda_status(e, "decode_attention_static: cudaGetSymbolAddress (error word)");
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_status(e, "decode_attention_static: SM count");
    s.sm_count = sms;
    s.err = static_cast<uint32_t*>(pe);
    s.partial = static_cast<float*>(p);
  }
  *out = s;
  return Status::ok();
}

Status decode_attention_static(const welvet_b200_mha_config& cfg_in, int batch, int max_ctx, const void* q,
                               int ldq, const void* k_pool, const void* v_pool, const int* block_table,
                               int max_pages, const int* ctx_len, void* out, int ldo, cudaStream_t stream) {
  if (batch <= 0 || max_ctx <= 0 || !q || !k_pool || !v_pool || !block_table || !ctx_len || !out ||
      (int64_t)max_pages * kPageTokens < max_ctx)
    return Status::err(1, "decode_attention_static: invalid argument");
  Cfg c;
  WV_TRY(resolve_config(cfg_in, &c));
  if (c.c.mask != 1)
    return Status::err(2, "decode_attention_static: only the causal mask (every cached key) is supported");
  const int heads = c.c.head_count;
  const int kv_heads = heads / c.group;
  const bool bf16 = c.c.precision == 1;
  const int hd = c.hd;
  if (!(hd == 64 || hd == 128 || (bf16 && hd == 256)))
    return Status::err(2, "decode_attention_static: head_dim must be 64 or 128 (or 256 in BF16)");
  if (!(c.group == 1 || c.group == 2 || c.group == 4 || c.group == 8))
    return Status::err(2, "decode_attention_static: heads per KV head must be 1, 2, 4 or 8");
  if (ldq < heads * hd || ldo < heads * hd)
    return Status::err(1, "decode_attention_static: ldq/ldo smaller than heads*head_dim");
  const size_t per_split = (size_t)batch * heads * (hd + 2);
  if (per_split > kStaticDecodeFloats)
    return Status::err(1, "decode_attention_static: batch*heads*(head_dim+2) exceeds the static scratch of " +
                              std::to_string(kStaticDecodeFloats) + " floats");

  int device = c.c.device;
  if (device < 0 && cudaGetDevice(&device) != cudaSuccess)
    return Status::err(4, "decode_attention_static: no current device");
  if (device >= kMaxDevices) return Status::err(1, "decode_attention_static: device ordinal too large");
  DeviceRestore restore_device;
  int cur = -1;
  WV_CUDA(cudaGetDevice(&cur), "cudaGetDevice");
  if (cur != device) WV_CUDA(cudaSetDevice(device), "cudaSetDevice");
  StaticSlot slot;
  WV_TRY(static_slot(device, &slot));

  DecodeArgs d;
  d.q = q;
  d.ldq = ldq;
  d.k_pool = k_pool;
  d.v_pool = v_pool;
  d.block_table = block_table;
  d.max_pages = max_pages;
  d.ctx_len = ctx_len;
  d.out = out;
  d.ldo = ldo;
  d.is_bf16 = bf16 ? 1 : 0;
  d.batch = batch;
  d.num_heads = heads;
  d.num_kv_heads = kv_heads;
  d.head_dim = hd;
  d.alibi = c.alibi;
  d.sigmoid = c.c.softmax == 1;
  d.head_base = c.c.head_begin;
  d.total_heads = c.c.num_heads;
  d.scale = c.scale;
  d.max_ctx = max_ctx;
  d.sm_count = slot.sm_count;
  d.partial = slot.partial;
  d.err = slot.err;
  const int want = decode_splits(d);
  d.splits = (int)std::min<size_t>((size_t)want, kStaticDecodeFloats / per_split);
  WV_CUDA(attn_decode(d, stream), "decode_attention_static");
  count_launch(2);
  return Status::ok();
}

}  // namespace

// Reads and clears g_decode_err of the current device when this entry point has
// run on it (no allocation: the word is this module's own variable).
Status take_static_decode_error(uint32_t* code) {
  *code = 0;
  int device = -1;
  WV_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) return Status::ok();
  {
    std::lock_guard<std::mutex> lock(g_slots_mu);
    if (!g_slots[device].err) return Status::ok();
  }
  WV_CUDA(cudaMemcpyFromSymbol(code, g_decode_err, sizeof(uint32_t)), "read static decode error word");
  if (*code) {
    const uint32_t zero = 0;
    WV_CUDA(cudaMemcpyToSymbol(g_decode_err, &zero, sizeof(uint32_t)), "clear static decode error word");
  }
  return Status::ok();
}

}  // namespace wv

// No counterpart in the reference; declared in include/welvet_b200.h.
extern "C" welvet_status welvet_b200_decode_attention_static(const welvet_b200_mha_config* cfg, int32_t batch,
                                                             int32_t max_ctx, const void* q, int32_t ldq,
                                                             const void* k_pool, const void* v_pool,
                                                             const int32_t* block_table, int32_t max_pages,
                                                             const int32_t* ctx_len, void* out, int32_t ldo,
                                                             void* stream) {
  if (!cfg) return wv::to_c(wv::Status::err(1, "decode_attention_static: invalid argument"));
  return wv::to_c(wv::decode_attention_static(*cfg, batch, max_ctx, q, ldq, k_pool, v_pool, block_table, max_pages,
                                              ctx_len, out, ldo, static_cast<cudaStream_t>(stream)));
}
