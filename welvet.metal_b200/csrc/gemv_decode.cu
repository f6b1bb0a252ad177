// Few-row BF16 projection of a decode step: out = x W^T for M <= 64 rows (one new
// token per sequence), the Dense forward of the reference's decode path
// (shaders/welvet_dense.metal:54-85 per output, src/layers/mha/mha.cpp:138-205 for
// the q/k/v and output projections), written for what bounds it on the B200: the
// weight matrix is read from HBM once, and at these sizes (a few to a hundred MB)
// the time is one memory round trip plus the transfer, so every load is issued up
// front and the M rows ride along on m16n8k16 tensor-core MMAs.
//
// Work split: a CTA (16 warps) owns 128 output columns over a 512-wide K slice;
// warp w owns the n8 tile of columns [8w, 8w + 8); a thread-block cluster of
// ks = K / 512 CTAs (at most 8) along K covers the whole K range. A thread issues
// its sixteen 16-byte W loads at once (row n = lane / 4, k = 32 q + 8 (lane % 4):
// four threads read 64 contiguous bytes of a row), while the CTA stages the x rows
// of its slice in shared memory. Each 32-wide k chunk is consumed by two k16 MMAs
// under a fixed permutation of k inside the chunk (logical k pairs {2c, 2c+1} /
// {2c+8, 2c+9} of MMA m are physical 8c + 4m + {0,1} / {2,3}); x and W use the
// same permutation, so the dot products are unchanged.
//
// Epilogue: each CTA writes its FP32 partial tile to shared memory; after a
// cluster barrier CTA r sums the partials of rows [r R, (r+1) R) from every CTA of
// the cluster in cluster-rank order (distributed shared memory, four columns per
// load; deterministic) and applies RoPE (rotate-half pairs inside a head: a head
// lies inside one 128-column tile for head_dim 32/64/128), then stores bf16 rows,
// with the K and V column ranges scattered into the KV page pools (the cache
// append) when kv_k is given.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace wv {
namespace {

constexpr int kThreads = 512;
constexpr int kNC = 128;         // output columns per CTA
constexpr int kSlice = 512;      // K per CTA
constexpr int kChunks = kSlice / 32;
constexpr int kRedLd = kNC + 4;  // padded row of the partial tile (floats)
constexpr int kXRow = kSlice * 2 + 16;  // bytes of a staged x row (pad: conflict-free fragment reads)
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
// Four floats of another CTA's shared memory (ordered by the cluster barriers
// around the reads; no clobber, so the loads of one sum are in flight together).
__device__ __forceinline__ float4 ld_dsmem_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1) gemv_decode_kernel(const VParams p) {
  extern __shared__ __align__(16) float vsm[];
  uint8_t* xs = reinterpret_cast<uint8_t*>(vsm);  // [16 MT][kXRow] x rows of the slice
  const int ks = p.ks;
  const int rank = ks > 1 ? (int)cluster_rank() : 0;
  const int tile = blockIdx.x / ks;
  const int n0 = tile * kNC;
  const int kbeg = rank * kSlice;
  const int warp = (int)warp_id(), lane = (int)lane_id(), tid = (int)threadIdx.x;
  const int g = lane >> 2, c = lane & 3;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);

  // Every W load of this thread, issued before anything waits.
  const int n = n0 + 8 * warp + g;
  const bool wok = n < p.N;
  const __nv_bfloat16* wr = p.w + (size_t)(wok ? n : 0) * p.K + kbeg + 8 * c;
  uint4 wv[kChunks];
#pragma unroll
  for (int q = 0; q < kChunks; ++q) wv[q] = wok ? ldg_stream_v4(wr + 32 * q) : zero;
  // The x rows of the slice into shared memory (rows past M as zeros).
  {
    constexpr int kUnits = MT * 16 * (kSlice / 8);  // 16-byte units
    uint4 xv[kUnits / kThreads];
#pragma unroll
    for (int i = 0; i < kUnits / kThreads; ++i) {
      const int u = tid + i * kThreads, row = u / (kSlice / 8), cu = u % (kSlice / 8);
      xv[i] = row < p.M ? ldg_nc_v4(p.x + (size_t)row * p.ldx + kbeg + 8 * cu) : zero;
    }
#pragma unroll
    for (int i = 0; i < kUnits / kThreads; ++i) {
      const int u = tid + i * kThreads, row = u / (kSlice / 8), cu = u % (kSlice / 8);
      *reinterpret_cast<uint4*>(xs + row * kXRow + 16 * cu) = xv[i];
    }
  }
  __syncthreads();
  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
  const uint8_t* xth = xs + g * kXRow + 16 * c;
#pragma unroll
  for (int q = 0; q < kChunks; ++q) {
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
      const uint8_t* xa_p = xth + (16 * mi) * kXRow + 64 * q;
      const uint4 xa = *reinterpret_cast<const uint4*>(xa_p);
      const uint4 xb = *reinterpret_cast<const uint4*>(xa_p + 8 * kXRow);
      mma_bf16_16816(acc[mi], xa.x, xb.x, xa.y, xb.y, wv[q].x, wv[q].y);
      mma_bf16_16816(acc[mi], xa.z, xb.z, xa.w, xb.w, wv[q].z, wv[q].w);
    }
  }
  __syncthreads();  // the x area becomes the partial tiles
  float* red = vsm;                     // [MT*16][kRedLd] this CTA's partial tile
  float* fin = vsm + MT * 16 * kRedLd;  // [MT*16][kRedLd] the summed rows of this CTA's slice
  // Partial tile: rows 16 mi + g (+8), columns 8 warp + 2 c (+1).
#pragma unroll
  for (int mi = 0; mi < MT; ++mi) {
    float* r0 = red + (16 * mi + g) * kRedLd + 8 * warp + 2 * c;
    *reinterpret_cast<float2*>(r0) = make_float2(acc[mi][0], acc[mi][1]);
    *reinterpret_cast<float2*>(r0 + 8 * kRedLd) = make_float2(acc[mi][2], acc[mi][3]);
  }
  // Rows of this CTA's slice, summed over the cluster in rank order. A thread
  // handles columns [4 (tid % 32), + 4) of rows tid / 32 + 16 it.
  const int rows = MT * 16;
  const int rpr = (rows + ks - 1) / ks;
  const int r0 = rank * rpr, r1 = min(rows, r0 + rpr);
  const int col = 4 * (tid % 32), rsub = tid / 32;
  if (ks > 1) {
    cluster_sync();  // every CTA's partial tile is written and visible
    uint32_t base[kMaxCluster];
#pragma unroll
    for (int q = 0; q < kMaxCluster; ++q) base[q] = q < ks ? dsmem_addr(red, (uint32_t)q) : 0u;
#pragma unroll
    for (int it = 0; it < MT; ++it) {
      const int row = rsub + 16 * it;
      if (row < r0 || row >= r1) continue;
      const uint32_t off = (uint32_t)((row * kRedLd + col) * 4);
      float4 v[kMaxCluster];
#pragma unroll
      for (int q = 0; q < kMaxCluster; ++q) v[q] = q < ks ? ld_dsmem_v4(base[q] + off) : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 sm = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kMaxCluster; ++q) {  // rank order (absent ranks add 0)
        sm.x += v[q].x;
        sm.y += v[q].y;
        sm.z += v[q].z;
        sm.w += v[q].w;
      }
      *reinterpret_cast<float4*>(fin + row * kRedLd + col) = sm;
    }
    cluster_sync();  // the other CTAs are done reading this CTA's partial tile
  } else {
    __syncthreads();
#pragma unroll
    for (int it = 0; it < MT; ++it) {
      const int row = rsub + 16 * it;
      *reinterpret_cast<float4*>(fin + row * kRedLd + col) = *reinterpret_cast<const float4*>(red + row * kRedLd + col);
    }
    __syncthreads();
  }
  // RoPE, then bf16 stores (q columns) or the KV page scatter (k, v columns); four
  // columns per thread stay inside one head (head_dim is a multiple of 4).
  const int hd = p.head_dim, half = hd >> 1;
  const int gc = n0 + col;
  if (gc >= p.N) return;
  const bool roped = gc < p.rope_cols;
  const int in_head = gc % hd;
  const bool to_kv = p.kv_k && gc >= p.kv_col0;
  int rel = gc - p.kv_col0;
  const bool is_v = to_kv && rel >= p.kv_dim;
  if (is_v) rel -= p.kv_dim;
  const int nk = p.kv_dim > 0 ? p.kv_dim / hd : 1;
  __nv_bfloat16* kv_base = is_v ? p.kv_v : p.kv_k;
  const int pcol = in_head < half ? col + half : col - half;  // rotate-half partner
#pragma unroll
  for (int it = 0; it < MT; ++it) {
    const int row = rsub + 16 * it;
    if (row < r0 || row >= r1 || row >= p.M) continue;
    float4 v = *reinterpret_cast<const float4*>(fin + row * kRedLd + col);
    if (roped) {
      const int pos = p.positions ? p.positions[row] : (p.pos_mod > 0 ? row % p.pos_mod : row);
      const bool pos_ok = pos >= 0 && pos < p.rope_max_pos;
      if (!pos_ok) atomicCAS(p.err, 0u, 0x100u);
      const float4 o = *reinterpret_cast<const float4*>(fin + row * kRedLd + pcol);
      float vv[4] = {v.x, v.y, v.z, v.w};
      const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 cs = pos_ok ? p.rope_tab[(size_t)pos * half + ((in_head + e) % half)] : make_float2(1.f, 0.f);
        vv[e] = in_head < half ? vv[e] * cs.x - ov[e] * cs.y : ov[e] * cs.y + vv[e] * cs.x;
      }
      v = make_float4(vv[0], vv[1], vv[2], vv[3]);
    }
    const uint2 pk = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    if (to_kv) {
      const int slot = p.kv_slot[row];
      if (slot < 0) continue;
      // pool layout [page][kv_head][kPageTokens][head_dim]
      const size_t off =
          (((size_t)(slot / kPageTokens) * nk + rel / hd) * kPageTokens + slot % kPageTokens) * hd + rel % hd;
      *reinterpret_cast<uint2*>(kv_base + off) = pk;
    } else {
      *reinterpret_cast<uint2*>(p.out + (size_t)row * p.ldo + gc) = pk;
    }
  }
}

// Shared memory: the staged x rows, later the partial and summed tiles.
template <int MT> constexpr int smem_bytes() {
  return std::max(MT * 16 * kXRow, 2 * MT * 16 * kRedLd * (int)sizeof(float));
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

}  // namespace

bool gemv_decode_supported(const GemmArgs& a) {
  if (a.kind != kGemmBF16 || !a.out_bf16 || a.a_lo || a.b_lo || a.out_hi || a.swiglu) return false;
  // K in whole 512-wide slices, at most kMaxCluster of them (one cluster along K)
  if (a.M < 1 || a.M > 64 || a.N < 4 || a.N % 4 || a.K < kSlice || a.K % kSlice || a.K / kSlice > kMaxCluster)
    return false;
  if (a.ldb != a.K || a.lda < a.K || a.lda % 8 || a.ldo % 4) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a.a) || !al16(a.b) || (reinterpret_cast<uintptr_t>(a.out) & 7)) return false;
  if (a.rope_cols > 0) {
    // a head lies inside one 128-column tile
    if (!a.rope_tab || !(a.head_dim == 32 || a.head_dim == 64 || a.head_dim == 128)) return false;
  }
  if (a.kv_k && (!a.kv_v || !a.kv_slot || a.head_dim <= 0 || a.head_dim % 4 || a.kv_dim % a.head_dim ||
                 (reinterpret_cast<uintptr_t>(a.kv_k) & 7) || (reinterpret_cast<uintptr_t>(a.kv_v) & 7)))
    return false;
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
  p.ks = a.K / kSlice;
  const int tiles = (a.N + kNC - 1) / kNC;
  switch ((a.M + 15) / 16) {
    case 1: return launch<1>(p, tiles, s);
    case 2: return launch<2>(p, tiles, s);
    case 3: return launch<3>(p, tiles, s);
    default: return launch<4>(p, tiles, s);
  }
}

}  // namespace wv
