// Few-row BF16 projection of a decode step: out = x W^T for M <= 64 rows (one new
// token per sequence), the Dense forward of the reference's decode path
// (shaders/welvet_dense.metal:54-85 per output, src/layers/mha/mha.cpp:138-205 for
// the q/k/v and output projections), written for what bounds it on the B200: the
// weight matrix is streamed from HBM once, so the kernel is a GEMV at HBM rate with
// the M rows riding along on m16n8k16 tensor-core MMAs.
//
// Work split: a CTA (8 warps) owns 128 output columns, warp w the 16 columns
// [16w, 16w + 16) as two n8 tiles, over a K slice; a thread-block cluster of ks
// CTAs along K covers the whole K range, one CTA per SM. The slice streams through a
// four-stage cp.async ring of 128-wide k steps (three steps, 96 KB of W, in flight
// per SM): per 32-wide k chunk a thread fetches 16 bytes of each of its two W rows
// (n = lane / 4, k = 8 (lane % 4) .. + 8: four threads read 64 contiguous bytes of a
// row) into its own slots, and the step's x rows go to a shared part of the stage.
// A chunk is consumed by two k16 MMAs under a fixed permutation of k inside the
// chunk (logical k pairs {2c, 2c+1} / {2c+8, 2c+9} of MMA m are physical
// 8c + 4m + {0,1} / {2,3}); x and W use the same permutation, so the dot products
// are unchanged.
//
// Epilogue: each CTA writes its FP32 partial tile to shared memory; after a
// cluster barrier CTA r sums the partials of rows [r R, (r+1) R) from every CTA of
// the cluster in cluster-rank order (distributed shared memory; deterministic) and
// applies RoPE (rotate-half pairs inside a head: a head lies inside one 128-column
// tile for head_dim 32/64/128), then stores bf16 rows, with the K and V column
// ranges scattered into the KV page pools (the cache append) when kv_k is given.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace wv {
namespace {

constexpr int kThreads = 256;
constexpr int kNC = 128;   // output columns per CTA
constexpr int kKU = 128;   // k per unrolled iteration (four 32-wide chunks)
constexpr int kRedLd = kNC + 4;  // padded row of the partial tile (floats)
constexpr int kMaxCluster = 8;

struct VParams {
  const __nv_bfloat16* x;
  int ldx;
  const __nv_bfloat16* w;
  int M, N, K, ks;
  __nv_bfloat16* out;
  int ldo;
  const float2* rope_tab;
  int rope_cols, head_dim, rope_max_pos;
  const int* positions;
  int pos_mod;
  __nv_bfloat16* kv_k;
  __nv_bfloat16* kv_v;
  const int* kv_slot;
  int kv_col0, kv_dim;
  uint32_t* err;
};

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// Weights are read once: no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// (ordered by the cluster barriers around the reads; no clobber, so the loads of
// one sum are in flight together)
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t n = pred ? 16u : 0u;  // 0 source bytes: the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}

// Stage s of the ring: each thread's eight 16-byte W fragments (four k chunks x two
// rows) at [q][j][thread] (a warp's reads hit consecutive 16-byte words), then the
// x rows of the step, [16 MT][128 k] with a 16-byte pad per row.
constexpr int kStages = 4;
constexpr int kWStage = 8 * kThreads * 16;  // 32 KB
constexpr int kXRow = kKU * 2 + 16;         // bytes of a staged x row
template <int MT> __host__ __device__ constexpr int stage_bytes() { return kWStage + MT * 16 * kXRow; }

template <int MT>
__global__ void __launch_bounds__(kThreads, 1) gemv_decode_kernel(const VParams p) {
  extern __shared__ __align__(16) float vsm[];
  uint8_t* ring = reinterpret_cast<uint8_t*>(vsm);
  const int ks = p.ks;
  const int rank = ks > 1 ? (int)cluster_rank() : 0;
  const int tile = blockIdx.x / ks;
  const int n0 = tile * kNC;
  const int kslice = p.K / ks, kbeg = rank * kslice;
  const int steps = kslice / kKU;
  const int warp = (int)warp_id(), lane = (int)lane_id(), tid = (int)threadIdx.x;
  const int g = lane >> 2, c = lane & 3;

  // This thread's two W rows (one per n8 tile) from column kbeg + 8c.
  const __nv_bfloat16* wr[2];
  bool wok[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int n = n0 + 16 * warp + 8 * j + g;
    wok[j] = n < p.N;
    wr[j] = p.w + (size_t)(wok[j] ? n : 0) * p.K + kbeg + 8 * c;
  }
  // Step i into its stage: this thread's W fragments and its share of the x rows.
  auto issue = [&](int i) {
    uint8_t* st = ring + (i % kStages) * stage_bytes<MT>();
    const int k0 = i * kKU;
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int j = 0; j < 2; ++j) cp_async16(st + ((q * 2 + j) * kThreads + tid) * 16, wr[j] + k0 + 32 * q, wok[j]);
    uint8_t* xs = st + kWStage;
#pragma unroll
    for (int u = tid; u < MT * 16 * 16; u += kThreads) {  // 16 units of 16 bytes per row
      const int row = u >> 4, cu = u & 15;
      const bool ok = row < p.M;
      cp_async16(xs + row * kXRow + 16 * cu, p.x + (size_t)(ok ? row : 0) * p.ldx + kbeg + k0 + 8 * cu, ok);
    }
  };
#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) {
    if (i < steps) issue(i);
    cp_async_commit();
  }
  float acc[MT][2][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

  for (int i = 0; i < steps; ++i) {
    cp_async_wait<kStages - 2>();  // this thread's copies of step i are complete
    __syncthreads();               // ... and every thread's (x rows); step i - 1 is consumed
    if (i + kStages - 1 < steps) issue(i + kStages - 1);
    cp_async_commit();
    const uint8_t* st = ring + (i % kStages) * stage_bytes<MT>();
    const uint8_t* xth = st + kWStage + g * kXRow + 16 * c;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 wv[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) wv[j] = *reinterpret_cast<const uint4*>(st + ((q * 2 + j) * kThreads + tid) * 16);
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        const uint8_t* xa_p = xth + (16 * mi) * kXRow + 64 * q;
        const uint4 xa = *reinterpret_cast<const uint4*>(xa_p);
        const uint4 xb = *reinterpret_cast<const uint4*>(xa_p + 8 * kXRow);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mma_bf16_16816(acc[mi][j], xa.x, xb.x, xa.y, xb.y, wv[j].x, wv[j].y);
          mma_bf16_16816(acc[mi][j], xa.z, xb.z, xa.w, xb.w, wv[j].z, wv[j].w);
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the x area becomes the partial tiles
  float* red = vsm;                        // [MT*16][kRedLd] this CTA's partial tile
  float* fin = vsm + MT * 16 * kRedLd;     // [MT*16][kRedLd] the summed rows of this CTA's slice
  // Partial tile: rows 16 i + g (+8), columns 16 warp + 8 j + 2 c (+1).
#pragma unroll
  for (int i = 0; i < MT; ++i) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int col = 16 * warp + 8 * j + 2 * c;
      float* r0 = red + (16 * i + g) * kRedLd + col;
      float* r1 = r0 + 8 * kRedLd;
      r0[0] = acc[i][j][0];
      r0[1] = acc[i][j][1];
      r1[0] = acc[i][j][2];
      r1[1] = acc[i][j][3];
    }
  }
  // Rows of this CTA's slice, summed over the cluster in rank order.
  const int rows = MT * 16;
  const int rpr = (rows + ks - 1) / ks;
  const int r0 = rank * rpr, r1 = min(rows, r0 + rpr);
  if (ks > 1) {
    cluster_sync();  // every CTA's partial tile is written and visible
    for (int e = threadIdx.x; e < (r1 - r0) * kNC; e += kThreads) {
      const int row = r0 + e / kNC, col = e % kNC;
      const float* loc = red + row * kRedLd + col;
      float v[kMaxCluster];
#pragma unroll
      for (int q = 0; q < kMaxCluster; ++q) v[q] = q < ks ? ld_dsmem_f32(dsmem_addr(loc, (uint32_t)q)) : 0.f;
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < kMaxCluster; ++q) s += v[q];  // rank order (absent ranks add 0)
      fin[row * kRedLd + col] = s;
    }
    cluster_sync();  // the other CTAs are done reading this CTA's partial tile
  } else {
    __syncthreads();
    for (int e = threadIdx.x; e < rows * kNC; e += kThreads) {
      const int row = e / kNC, col = e % kNC;
      fin[row * kRedLd + col] = red[row * kRedLd + col];
    }
    __syncthreads();
  }
  // RoPE, then bf16 stores (q columns) or the KV page scatter (k, v columns).
  const int hd = p.head_dim, half = hd >> 1;
  for (int e = threadIdx.x; e < (r1 - r0) * kNC; e += kThreads) {
    const int row = r0 + e / kNC, col = e % kNC, gc = n0 + col;
    if (row >= p.M || gc >= p.N) continue;
    float v = fin[row * kRedLd + col];
    if (gc < p.rope_cols) {
      const int in_head = gc % hd;
      const int pos = p.positions ? p.positions[row] : (p.pos_mod > 0 ? row % p.pos_mod : row);
      const bool pos_ok = pos >= 0 && pos < p.rope_max_pos;
      if (!pos_ok) atomicCAS(p.err, 0u, 0x100u);
      const float2 cs = pos_ok ? p.rope_tab[(size_t)pos * half + (in_head % half)] : make_float2(1.f, 0.f);
      if (in_head < half) {
        const float b = fin[row * kRedLd + col + half];
        v = v * cs.x - b * cs.y;
      } else {
        const float a = fin[row * kRedLd + col - half];
        v = a * cs.y + v * cs.x;
      }
    }
    if (p.kv_k && gc >= p.kv_col0) {
      int rel = gc - p.kv_col0;
      const bool is_v = rel >= p.kv_dim;
      if (is_v) rel -= p.kv_dim;
      const int slot = p.kv_slot[row];
      if (slot < 0) continue;
      // pool layout [page][kv_head][kPageTokens][head_dim]
      const int nk = p.kv_dim / hd;
      const size_t off =
          (((size_t)(slot / kPageTokens) * nk + rel / hd) * kPageTokens + slot % kPageTokens) * hd + rel % hd;
      (is_v ? p.kv_v : p.kv_k)[off] = __float2bfloat16_rn(v);
    } else {
      p.out[(size_t)row * p.ldo + gc] = __float2bfloat16_rn(v);
    }
  }
}

// Shared memory: the ring, later the partial and summed tiles.
template <int MT> constexpr int smem_bytes() {
  return std::max(kStages * stage_bytes<MT>(), 2 * MT * 16 * kRedLd * (int)sizeof(float));
}

template <int MT>
cudaError_t launch(const VParams& p, int tiles, cudaStream_t s) {
  auto kern = gemv_decode_kernel<MT>;
  constexpr int smem = smem_bytes<MT>();
  static const cudaError_t ready = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (ready != cudaSuccess) return ready;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(tiles * p.ks, 1, 1);
  lc.blockDim = dim3(kThreads, 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = p.ks;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, kern, p);
}

// Cluster size along K: the largest that keeps the grid within one CTA per SM
// (one wave), the K slice a whole number of 128-wide steps.
int cluster_size(int tiles, int K, int sm_count) {
  int best = 1;
  for (int ks = 2; ks <= kMaxCluster; ks *= 2) {
    if (K % (kKU * ks) || tiles * ks > sm_count) break;
    best = ks;
  }
  return best;
}

}  // namespace

bool gemv_decode_supported(const GemmArgs& a) {
  if (a.kind != kGemmBF16 || !a.out_bf16 || a.a_lo || a.b_lo || a.out_hi || a.swiglu) return false;
  if (a.M < 1 || a.M > 64 || a.N < 1 || a.K < kKU || a.K % kKU) return false;
  if (a.ldb != a.K || a.lda < a.K || a.lda % 8) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a.a) || !al16(a.b)) return false;
  if (a.rope_cols > 0) {
    // a head lies inside one 128-column tile
    if (!a.rope_tab || !(a.head_dim == 32 || a.head_dim == 64 || a.head_dim == 128)) return false;
  }
  if (a.kv_k && (!a.kv_v || !a.kv_slot || a.head_dim <= 0 || a.kv_dim % a.head_dim)) return false;
  return true;
}

cudaError_t gemv_decode(const GemmArgs& a, cudaStream_t s) {
  if (!gemv_decode_supported(a)) return cudaErrorInvalidValue;
  VParams p{};
  p.x = static_cast<const __nv_bfloat16*>(a.a);
  p.ldx = a.lda;
  p.w = static_cast<const __nv_bfloat16*>(a.b);
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.ldo = a.ldo;
  p.rope_tab = a.rope_tab;
  p.rope_cols = a.rope_cols;
  p.head_dim = a.head_dim > 0 ? a.head_dim : 64;
  p.rope_max_pos = a.rope_max_pos;
  p.positions = a.positions;
  p.pos_mod = a.pos_mod;
  p.kv_k = static_cast<__nv_bfloat16*>(a.kv_k);
  p.kv_v = static_cast<__nv_bfloat16*>(a.kv_v);
  p.kv_slot = a.kv_slot;
  p.kv_col0 = a.kv_col0;
  p.kv_dim = a.kv_dim;
  p.err = a.err;
  const int tiles = (a.N + kNC - 1) / kNC;
  p.ks = cluster_size(tiles, a.K, a.sm_count);
  switch ((a.M + 15) / 16) {
    case 1: return launch<1>(p, tiles, s);
    case 2: return launch<2>(p, tiles, s);
    case 3: return launch<3>(p, tiles, s);
    default: return launch<4>(p, tiles, s);
  }
}

}  // namespace wv
