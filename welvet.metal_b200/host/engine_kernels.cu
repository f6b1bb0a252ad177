// Small bookkeeping kernels of the KV cache (slots, positions, lengths).
// Kept on the device so a decode step needs no host->device traffic.
#include "engine.hpp"

namespace wv {
namespace {

__global__ void prefill_slots_kernel(int* slots, int batch, int seq, int pps) {
  const int64_t n = (int64_t)batch * seq;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / seq), t = (int)(i % seq);
    slots[i] = b * pps * kPageTokens + t;
  }
}

__global__ void decode_rows_kernel(int* ctx, int* positions, int* slots, int batch, int pps) {
  // the next kernel (the q/k/v projection) may start loading its weights
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int L = ctx[b];
  positions[b] = L;
  slots[b] = b * pps * kPageTokens + L;
  ctx[b] = L + 1;
}

__global__ void set_ctx_kernel(int* ctx, int batch, int value) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) ctx[b] = value;
}

__global__ void block_table_kernel(int* bt, int batch, int pps) {
  const int64_t n = (int64_t)batch * pps;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    bt[i] = (int)i;  // sequence b owns pages [b*pps, (b+1)*pps)
}

int blocks(int64_t n) { return (int)std::min<int64_t>((n + 255) / 256, 4096); }

} // namespace

cudaError_t make_prefill_slots(int* slots, int batch, int seq, int pps, cudaStream_t s) {
  prefill_slots_kernel<<<blocks((int64_t)batch * seq), 256, 0, s>>>(slots, batch, seq, pps);
  return cudaGetLastError();
}
cudaError_t make_decode_rows(int* ctx, int* positions, int* slots, int batch, int pps, cudaStream_t s) {
  decode_rows_kernel<<<(batch + 127) / 128, 128, 0, s>>>(ctx, positions, slots, batch, pps);
  return cudaGetLastError();
}
cudaError_t set_ctx(int* ctx, int batch, int value, cudaStream_t s) {
  set_ctx_kernel<<<(batch + 127) / 128, 128, 0, s>>>(ctx, batch, value);
  return cudaGetLastError();
}
cudaError_t make_block_table(int* bt, int batch, int pps, cudaStream_t s) {
  block_table_kernel<<<blocks((int64_t)batch * pps), 256, 0, s>>>(bt, batch, pps);
  return cudaGetLastError();
}

} // namespace wv
