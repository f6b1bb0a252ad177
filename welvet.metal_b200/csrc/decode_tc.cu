// Split-KV decode attention over the paged KV cache (BF16) for sm_100a.
//
// One new query per sequence attends over its cached keys: for a (sequence, KV
// head, split) the CTA streams the split's pages of K and V and the G query heads
// of the KV group share every byte read, so the kernel is HBM-bound. Data path:
//   * each of the 4 warps owns a ring of page stages in shared memory; its lane 0
//     looks up the page in the block table and issues TMA tile loads (16 keys x 64
//     dims boxes, 128-byte swizzle) for K and V, completing on the stage mbarrier;
//     warp w takes pages w, w+4, w+8, ... of the split;
//   * the G (<= 8) query rows sit in the A fragment of m16n8k16 BF16 MMAs
//     (rows >= G are zero): S = Q K^T per page with K^T fragments read by ldmatrix
//     from the swizzled stage, online softmax in the log2 domain on the S fragment
//     (row max / sum over the 4 lanes of a row by two shuffles), then O += P V with
//     P reused from the S fragment as the A operand and V^T fragments from
//     ldmatrix.trans;
//   * the four warps' (m, l, O) merge through shared memory into the split's
//     partial slot [B, NH, splits, head_dim + 2], which decode_combine_kernel
//     (attn_simt.cu) reduces over splits, as for the CUDA-core decode kernel.
// The MMAs are a small fraction of the time; they replace the per-key shuffle
// reductions of a CUDA-core dot product. Every wait is bounded (WV_WAIT_LIMIT_NS).
// Reference semantics: shaders/ops_mha.metal:31-127 with one query row at position
// ctx_len - 1 (causal over the whole cache), ALiBi and sigmoid variants included.
#include "common.cuh"
#include "kernels.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>

namespace wv {
namespace {

constexpr int kWarps = 4;
constexpr int kBox = 64;                       // dims per TMA box (128 bytes of BF16)
constexpr int kBoxBytes = kPageTokens * 128;   // one 16-row box

template <int HD> struct DT {
  static constexpr int NBOX = HD / kBox;
  static constexpr int TILE = NBOX * kBoxBytes;                   // one page of K (or V)
  static constexpr int STAGES = HD == 256 ? 2 : 3;  // per warp
  static constexpr int STAGE_BYTES = 2 * TILE;                     // K + V
  static constexpr int RING = STAGES * STAGE_BYTES;                // per warp
  static constexpr int OFF_BAR = kWarps * RING;
  static constexpr int SMEM = 1024 + OFF_BAR + kWarps * STAGES * 8 + 64;
  static_assert(kWarps * 8 * (HD + 2) * 4 <= kWarps * RING, "merge area must fit in the rings");
};

WV_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
WV_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D = A B + D, m16n8k16, BF16 inputs, FP32 accumulators. A rows 8..15 are zero here,
// so a1 = a3 = 0 and d2, d3 stay 0.
WV_DEV void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
// Byte offset of (row, 16-byte chunk c of the full head_dim row) in a page tile
// written by 64-dim TMA boxes with the 128-byte swizzle.
WV_DEV uint32_t tile_off(int row, int c) {
  return (uint32_t)((c >> 3) * kBoxBytes + row * 128 + (((c & 7) ^ (row & 7)) << 4));
}

template <int HD, int G, bool ALIBI, bool SIGMOID>
__global__ void __launch_bounds__(kWarps * 32)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const DecodeArgs a, int splits, int chunk) {
  using D = DT<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = (int)warp_id(), lane = (int)lane_id();
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + D::OFF_BAR) + warp * D::STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + D::OFF_BAR + kWarps * D::STAGES * 8);
  uint32_t* local_err = reinterpret_cast<uint32_t*>(smem + D::OFF_BAR + kWarps * D::STAGES * 8 + 4);
  uint32_t* err = a.err ? a.err : local_err;
  uint8_t* ring = smem + warp * D::RING;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    *local_err = 0;
  }
  if (lane == 0)
    for (int s = 0; s < D::STAGES; ++s) mbar_init(&full[s], 1);
  fence_barrier_init();
  __syncthreads();
  // Launched as a programmatic dependent of the q/k/v projection: the lengths, q and
  // the step's appended K/V row are read only after it has completed; the combine
  // kernel behind this one may launch now (it waits the same way).
  pdl_wait();
  pdl_trigger();

  const int L = a.ctx_len[b];
  const int k0 = split * chunk, k1 = min(L, k0 + chunk);
  const int pg0 = k0 / kPageTokens;
  const int npages = k1 > k0 ? (k1 - k0 + kPageTokens - 1) / kPageTokens : 0;
  const int mine = npages > warp ? (npages - warp + kWarps - 1) / kWarps : 0;  // pages of this warp

  const int* bt = a.block_table + (size_t)b * a.max_pages;
  auto issue = [&](int i) {  // lane 0: page i of this warp into stage i % STAGES
    const int s = i % D::STAGES;
    const int page = bt[pg0 + warp + kWarps * i];
    const int row = (page * a.num_kv_heads + kh) * kPageTokens;
    uint8_t* kt = ring + s * D::STAGE_BYTES;
    uint8_t* vt = kt + D::TILE;
    mbar_arrive_expect_tx(&full[s], D::STAGE_BYTES);
#pragma unroll
    for (int x = 0; x < D::NBOX; ++x) {
      tma_load_2d(kt + x * kBoxBytes, &tmK, &full[s], x * kBox, row);
      tma_load_2d(vt + x * kBoxBytes, &tmV, &full[s], x * kBox, row);
    }
  };
  if (lane == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    for (int i = 0; i < min(mine, D::STAGES); ++i) issue(i);
  }

  // Q rows of the KV group as the A fragment (row g = lane / 4 < G), per 16 dims.
  const int g = lane >> 2, t = lane & 3;
  const int h = kh * G + g;  // query head of this lane's row (valid when g < G)
  uint32_t qa0[HD / 16], qa2[HD / 16];
  {
    const __nv_bfloat16* Q = static_cast<const __nv_bfloat16*>(a.q) + (size_t)b * a.ldq + (size_t)h * HD;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      qa0[kk] = g < G ? *reinterpret_cast<const uint32_t*>(Q + 16 * kk + 2 * t) : 0u;
      qa2[kk] = g < G ? *reinterpret_cast<const uint32_t*>(Q + 16 * kk + 8 + 2 * t) : 0u;
    }
  }
  const float qs = a.scale * 1.4426950408889634f;  // scores in the log2 domain
  const float slope2 = ALIBI && g < G
                           ? exp2f(-(float)(a.head_base + h + 1) * 8.0f / (float)a.total_heads) * 1.4426950408889634f
                           : 0.f;

  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool ok = true;

  const uint32_t ring_u32 = smem_u32(ring);
  for (int i = 0; i < mine; ++i) {
    const int s = i % D::STAGES;
    ok = mbar_wait(&full[s], (uint32_t)((i / D::STAGES) & 1), abort_flag, err, kErrWaitFull);
    if (!__all_sync(0xffffffffu, ok)) {
      ok = false;
      break;
    }
    const uint32_t kt = ring_u32 + s * D::STAGE_BYTES, vt = kt + D::TILE;
    const int kbase = (pg0 + warp + kWarps * i) * kPageTokens;  // position of key 0 of the page
    if (kbase + kPageTokens > k1) {
      // Last page of the range: its rows at and after k1 hold whatever the pool had
      // (possibly never written, NaN or Inf bit patterns). Their P is 0, but 0 * Inf
      // is NaN in the PV product, so the V rows are cleared first (K rows are
      // harmless: their scores are replaced by -inf).
      const int first = k1 - kbase;
      uint8_t* vrow = ring + s * D::STAGE_BYTES + D::TILE;
      for (int idx = lane; idx < (kPageTokens - first) * D::NBOX * 8; idx += 32) {
        const int r = first + idx / (D::NBOX * 8), x = (idx / 8) % D::NBOX, c = idx % 8;
        *reinterpret_cast<uint4*>(vrow + x * kBoxBytes + r * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }

    // ---- S = Q K^T for the 16 keys of the page (two n8 tiles)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      // matrix l/8: keys (l/16)*8 + l%8, 16-byte chunk 2kk + (l/8)%2
      const int key = ((lane >> 4) << 3) + (lane & 7);
      const int csub = (lane >> 3) & 1;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kt + tile_off(key, 2 * kk + csub), b0, b1, b2, b3);
        mma_bf16(sc[0], qa0[kk], qa2[kk], b0, b1);
        mma_bf16(sc[1], qa0[kk], qa2[kk], b2, b3);
      }
    }
    // ---- online softmax on row g: this lane holds keys 2t, 2t+1 (tile 0) and
    //      8+2t, 8+2t+1 (tile 1)
    float p[4];
    {
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = (e >> 1) * 8 + 2 * t + (e & 1);
        const int pos = kbase + key;
        float v = sc[e >> 1][e & 1] * qs;
        if (ALIBI) v -= slope2 * (float)((L - 1) - pos);
        x[e] = pos < k1 ? v : -INFINITY;
      }
      if (SIGMOID) {
#pragma unroll
        for (int e = 0; e < 4; ++e) p[e] = x[e] == -INFINITY ? 0.f : 1.f / (1.f + exp2f(-x[e]));
      } else {
        float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mnew = fmaxf(m, mx);
        const float mref = mnew == -INFINITY ? 0.f : mnew;
        const float corr = exp2f(m - mref);  // m = -inf -> 0 (nothing accumulated yet)
#pragma unroll
        for (int e = 0; e < 4; ++e) p[e] = exp2f(x[e] - mref);
        l = l * corr + ((p[0] + p[1]) + (p[2] + p[3]));
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
          o[j][0] *= corr;
          o[j][1] *= corr;
        }
        m = mnew;
      }
    }
    // ---- O += P V: P from the S fragment as the A operand (rows >= 8 zero)
    const uint32_t pa0 = pack_bf16x2(p[0], p[1]), pa2 = pack_bf16x2(p[2], p[3]);
    {
      // matrix l/8: keys ((l/8)&1)*8 + l%8, dims chunk j + l/16 (transposed load)
      const int key = (((lane >> 3) & 1) << 3) + (lane & 7);
      const int cadd = lane >> 4;
#pragma unroll
      for (int j = 0; j < HD / 8; j += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vt + tile_off(key, j + cadd), b0, b1, b2, b3);
        mma_bf16(o[j], pa0, pa2, b0, b1);
        mma_bf16(o[j + 1], pa0, pa2, b2, b3);
      }
    }
    // stage s is consumed: the warp's reads are complete before lane 0 refills it
    __syncwarp();
    if (lane == 0 && i + D::STAGES < mine) {
      fence_proxy_async_smem();
      issue(i + D::STAGES);
    }
  }
  // Row sum over the four lanes of the row.
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  // ---- merge the warps (the rings are free once every warp has left its loop)
  __syncthreads();
  if (!__syncthreads_and(ok ? 1 : 0)) return;  // a bounded wait gave up: error recorded
  float* mw = reinterpret_cast<float*>(smem);      // [kWarps][8]
  float* lw = mw + kWarps * 8;                     // [kWarps][8]
  float* ow = lw + kWarps * 8;                     // [kWarps][8][HD]
  if (g < G) {
    if (t == 0) {
      mw[warp * 8 + g] = SIGMOID ? 0.f : m;
      lw[warp * 8 + g] = l;
    }
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      ow[(warp * 8 + g) * HD + 8 * j + 2 * t] = o[j][0];
      ow[(warp * 8 + g) * HD + 8 * j + 2 * t + 1] = o[j][1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * (HD + 2); idx += blockDim.x) {
    const int r = idx / (HD + 2), c = idx % (HD + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w * 8 + r]);
    float val = 0.f;
    if (c == HD) {
      val = M;
    } else {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mwv = mw[w * 8 + r];
        const float wt = SIGMOID ? 1.f : (mwv == -INFINITY ? 0.f : exp2f(mwv - M));
        val += wt * (c < HD ? ow[(w * 8 + r) * HD + c] : lw[w * 8 + r]);
      }
    }
    a.partial[(((size_t)b * a.num_heads + kh * G + r) * splits + split) * (HD + 2) + c] = val;
  }
}

template <int HD, int G>
cudaError_t launch_g(const CUtensorMap& mk, const CUtensorMap& mv, const DecodeArgs& a, int splits, int chunk,
                     cudaStream_t s) {
  using D = DT<HD>;
  const dim3 grid(splits, a.num_kv_heads, a.batch);
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, D::SMEM);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, dim3(kWarps * 32), D::SMEM, s, mk, mv, a, splits, chunk);
  };
  if (a.sigmoid) return a.alibi ? go(decode_tc_kernel<HD, G, true, true>) : go(decode_tc_kernel<HD, G, false, true>);
  return a.alibi ? go(decode_tc_kernel<HD, G, true, false>) : go(decode_tc_kernel<HD, G, false, false>);
}

template <int HD>
cudaError_t launch_hd(const CUtensorMap& mk, const CUtensorMap& mv, const DecodeArgs& a, int G, int splits,
                      int chunk, cudaStream_t s) {
  switch (G) {
  case 1: return launch_g<HD, 1>(mk, mv, a, splits, chunk, s);
  case 2: return launch_g<HD, 2>(mk, mv, a, splits, chunk, s);
  case 4: return launch_g<HD, 4>(mk, mv, a, splits, chunk, s);
  case 8: return launch_g<HD, 8>(mk, mv, a, splits, chunk, s);
  default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int decode_tc_ctas_per_sm(int head_dim) {
  const int smem = head_dim == 64 ? DT<64>::SMEM : head_dim == 128 ? DT<128>::SMEM : DT<256>::SMEM;
  return std::max(1, (228 * 1024) / (smem + 1024));  // 1 KB of each CTA's shared memory is reserved
}

bool decode_tc_supported(const DecodeArgs& a) {
  if (!a.is_bf16 || a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads) return false;
  const int G = a.num_heads / a.num_kv_heads;
  if (!(G == 1 || G == 2 || G == 4 || G == 8)) return false;
  if (!(a.head_dim == 64 || a.head_dim == 128 || a.head_dim == 256)) return false;
  if (a.ldq % 8) return false;  // 16-byte aligned query rows (4-byte fragment loads)
  const uintptr_t kp = reinterpret_cast<uintptr_t>(a.k_pool), vp = reinterpret_cast<uintptr_t>(a.v_pool);
  return kp % 16 == 0 && vp % 16 == 0 && reinterpret_cast<uintptr_t>(a.q) % 4 == 0;
}

// Launches decode_tc_kernel for the splits of decode_splits(a) (chunks rounded up to
// whole pages); decode_combine_kernel follows in attn_decode.
cudaError_t attn_decode_tc(const DecodeArgs& a, int splits, cudaStream_t s) {
  const int G = a.num_heads / a.num_kv_heads;
  const int chunk = ((a.max_ctx + splits - 1) / splits + kPageTokens - 1) / kPageTokens * kPageTokens;
  // Pools viewed as [rows = pages * kv_heads * 16, head_dim]; a larger extent than the
  // pool is harmless (only block-table pages are addressed).
  const uint64_t rows = a.pool_rows > 0 ? (uint64_t)a.pool_rows : (uint64_t)1 << 30;
  alignas(64) CUtensorMap mk, mv;
  constexpr int kBf16 = (int)CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  constexpr int kSw128 = (int)CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_tma_2d(&mk, a.k_pool, kBf16, 2, a.head_dim, rows, a.head_dim, kBox, kPageTokens, kSw128) ||
      !make_tma_2d(&mv, a.v_pool, kBf16, 2, a.head_dim, rows, a.head_dim, kBox, kPageTokens, kSw128))
    return cudaErrorInvalidValue;
  switch (a.head_dim) {
  case 64: return launch_hd<64>(mk, mv, a, G, splits, chunk, s);
  case 128: return launch_hd<128>(mk, mv, a, G, splits, chunk, s);
  case 256: return launch_hd<256>(mk, mv, a, G, splits, chunk, s);
  default: return cudaErrorInvalidValue;
  }
}

}  // namespace wv
