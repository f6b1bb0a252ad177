// One-shot all-reduce of a small vector over NVLink peer memory (the output of a
// head-sharded decode step: batch x d_model partial sums per rank), in place of an
// NCCL all-reduce whose fixed latency (tens of microseconds at 8 ranks) is several
// times the transfer. The reference is single-device and has no counterpart.
//
// Every rank owns a receive area with one slot per sender and two parities, mapped
// into every other rank's address space (CUDA IPC). One launch per call, kPeerCtas
// CTAs, CTA c owning a contiguous piece of the vector:
//   1. push: CTA c writes its piece of the local partial into slot[rank] of every
//      rank's area (NVLink stores to the peers, plain stores to itself);
//   2. publish: after a system-scope fence, a release store of the call's epoch into
//      flag[parity][rank][c] of every rank;
//   3. wait: CTA c waits (bounded by time) until flag[parity][q][c] of its own area
//      holds the epoch for every sender q;
//   4. reduce: out = sum over q = 0 .. n-1 of slot[q], in rank order, so every rank
//      computes bit-identical sums.
// Epochs increase by one per call on every rank (all ranks call in the same order),
// and the parity alternates, so a slot is rewritten two calls later at the earliest:
// by then its reader has finished (the writer has seen the reader's flags of the
// call in between, which the reader publishes only after its previous call ended).
// A wait that runs out records kErrPeerWait in the error word and the CTA skips its
// reduction; nothing traps.
//
// peer_rs_sum is the owner's half of the prefill output's reduce-scatter, whose
// transfers are copy-engine copies (host/comm.cpp): it waits for the peers' epoch
// flags and sums the slices.
#include "common.cuh"
#include "kernels.h"

namespace wv {
namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(const PeerArgs a) {
  pdl_wait();  // launched as a programmatic dependent of the kernel producing `in`
  const int n = a.nranks, par = (int)(a.epoch & 1u), cta = blockIdx.x;
  // 16-byte units of the vector, split over the CTAs
  const size_t units = (a.count * (BF16 ? 2 : 4) + 15) / 16;
  const size_t per = (units + gridDim.x - 1) / gridDim.x;
  const size_t u0 = (size_t)cta * per, u1 = min(units, u0 + per);
  const uint4* src = static_cast<const uint4*>(a.in);
  // 1. push this CTA's piece into slot[par][rank] of every rank
  for (int p = 0; p < n; ++p) {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(a.areas[p]) +
                                          ((size_t)par * n + a.rank) * a.slot_bytes);
    for (size_t u = u0 + threadIdx.x; u < u1; u += kThreads) dst[u] = src[u];
  }
  __syncthreads();
  // 2. publish: flag[par][rank][cta] = epoch on every rank. The barrier orders the
  // CTA's stores before the flag writers' system-scope fence and release stores.
  if (threadIdx.x < (unsigned)n) {
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(static_cast<char*>(a.areas[threadIdx.x]) + a.flags_off);
    st_release_sys(f + ((size_t)par * n + a.rank) * gridDim.x + cta, a.epoch);
  }
  // 3. wait for every sender's piece of this CTA
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  if (threadIdx.x < (unsigned)n) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(static_cast<const char*>(a.areas[a.rank]) + a.flags_off) +
                        ((size_t)par * n + threadIdx.x) * gridDim.x + cta;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) != a.epoch) {
      if (globaltimer() - t0 > a.wait_ns) {
        atomicCAS(a.err, 0u, (uint32_t)kErrPeerWait);
        ok_all = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (!ok_all) return;
  // 4. reduce in rank order
  const char* own = static_cast<const char*>(a.areas[a.rank]) + (size_t)par * n * a.slot_bytes;
  uint4* out = static_cast<uint4*>(a.out);
  for (size_t u = u0 + threadIdx.x; u < u1; u += kThreads) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int q = 0; q < n; ++q) {
      const uint4 v = reinterpret_cast<const uint4*>(own + (size_t)q * a.slot_bytes)[u];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      if (BF16) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[2 * e] += __uint_as_float(w[e] << 16);
          acc[2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] += __uint_as_float(w[e]);
      }
    }
    if (BF16) {
      out[u] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                          pack_bf16x2(acc[6], acc[7]));
    } else {
      out[u] = make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                          __float_as_uint(acc[3]));
    }
  }
}

// Owner side of the chunked reduce-scatter: the N - 1 peers' slices of this rank's
// rows arrive by copy-engine transfers, each followed by a 4-byte epoch write into
// flag[q]; once every flag holds the epoch the rows are summed in rank order (this
// rank's own partial in place) and written over the own partial.
template <bool BF16>
__global__ void __launch_bounds__(256) peer_rs_sum_kernel(const PeerRsArgs a) {
  __shared__ int ok_all;
  if (threadIdx.x == 0) {
    ok_all = 1;
    const uint64_t t0 = globaltimer();
    for (int q = 0; q < a.nranks && ok_all; ++q) {
      if (q == a.rank) continue;
      while (ld_acquire_sys(a.flags + q) != a.epoch) {
        if (globaltimer() - t0 > a.wait_ns) {
          atomicCAS(a.err, 0u, (uint32_t)kErrPeerWait);
          ok_all = 0;
          break;
        }
        __nanosleep(2000);
      }
    }
  }
  __syncthreads();
  if (!ok_all) return;
  const size_t units = a.count * (BF16 ? 2 : 4) / 16;
  uint4* own = static_cast<uint4*>(a.own);
  for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < units; u += (size_t)gridDim.x * blockDim.x) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int q = 0; q < a.nranks; ++q) {
      const uint4 v = q == a.rank ? own[u]
                                  : reinterpret_cast<const uint4*>(static_cast<const char*>(a.slots) +
                                                                   (size_t)q * a.slot_bytes)[u];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      if (BF16) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[2 * e] += __uint_as_float(w[e] << 16);
          acc[2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] += __uint_as_float(w[e]);
      }
    }
    if (BF16) {
      own[u] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                          pack_bf16x2(acc[6], acc[7]));
    } else {
      own[u] = make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                          __float_as_uint(acc[3]));
    }
  }
}

// Receiving side of the attention-output exchange (output mode 2): the peers'
// column blocks of this rank's rows arrive by copy-engine transfers, each followed by
// a 4-byte epoch write into flags[q]. One warp, lane q waiting (bounded by time) for
// sender q, so the output projection queued behind this kernel on the same stream
// starts only once every block has landed. The kernel holds one SM for the wait only;
// the data needs no further pass.
__global__ void __launch_bounds__(32) peer_flags_wait_kernel(const uint32_t* flags, int nranks, int rank,
                                                             uint32_t epoch, uint64_t wait_ns, uint32_t* err) {
  const int q = (int)threadIdx.x;
  if (q >= nranks || q == rank) return;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flags + q) != epoch) {
    if (globaltimer() - t0 > wait_ns) {
      atomicCAS(err, 0u, (uint32_t)kErrPeerWait);
      return;
    }
    __nanosleep(500);
  }
}

}  // namespace

cudaError_t peer_flags_wait(const uint32_t* flags, int nranks, int rank, uint32_t epoch, uint64_t wait_ns,
                            uint32_t* err, cudaStream_t s) {
  if (!flags || !err || nranks < 2 || nranks > kPeerMaxRanks || rank < 0 || rank >= nranks)
    return cudaErrorInvalidValue;
  peer_flags_wait_kernel<<<1, 32, 0, s>>>(flags, nranks, rank, epoch, wait_ns, err);
  return cudaGetLastError();
}

cudaError_t peer_rs_sum(const PeerRsArgs& a, int grid, cudaStream_t s) {
  if (a.nranks < 2 || a.nranks > kPeerMaxRanks || a.rank < 0 || a.rank >= a.nranks || !a.own || !a.slots ||
      !a.flags || (reinterpret_cast<uintptr_t>(a.own) & 15) || (reinterpret_cast<uintptr_t>(a.slots) & 15) ||
      (a.count * (a.bf16 ? 2 : 4)) % 16 || a.count * (a.bf16 ? 2 : 4) > a.slot_bytes || grid < 1)
    return cudaErrorInvalidValue;
  if (a.bf16) peer_rs_sum_kernel<true><<<grid, 256, 0, s>>>(a);
  else peer_rs_sum_kernel<false><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t peer_allreduce(const PeerArgs& a, cudaStream_t s) {
  if (a.nranks < 1 || a.nranks > kPeerMaxRanks || a.rank < 0 || a.rank >= a.nranks || !a.in || !a.out ||
      (reinterpret_cast<uintptr_t>(a.in) & 15) || (reinterpret_cast<uintptr_t>(a.out) & 15))
    return cudaErrorInvalidValue;
  const size_t bytes = a.count * (a.bf16 ? 2 : 4);
  if (bytes % 16 || bytes > a.slot_bytes) return cudaErrorInvalidValue;
  return a.bf16 ? launch_pdl(peer_allreduce_kernel<true>, dim3(kPeerCtas), dim3(kThreads), 0, s, a)
                : launch_pdl(peer_allreduce_kernel<false>, dim3(kPeerCtas), dim3(kThreads), 0, s, a);
}

}  // namespace wv
