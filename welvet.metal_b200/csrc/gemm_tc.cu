// Projection GEMMs of the MHA forward (the Q/K/V and O Dense layers,
// src/layers/mha/mha.cpp:168-198, whose reference kernel is the one-thread-per-
// output soft-double GEMV shaders/welvet_dense.metal:54-85) as a persistent,
// warp-specialised tcgen05 GEMM for sm_100a:
//   warp 0      TMA producer (one elected thread) filling a ring of smem stages
//   warp 1      UMMA issuer (one thread); owns the TMEM allocation
//   warps 2-5   epilogue: TMEM -> registers -> (RoPE) -> global, one row per thread
//   warps 6..   (FP8: 8 warps, NF4: 16) dequantise B codes into a BF16 smem tile per stage
// Accumulators are double-buffered in TMEM so the epilogue of tile i overlaps the
// mainloop of tile i+1. Tiles: 128 x BN, K-blocks of 128 bytes per operand row
// (128-byte swizzle, the canonical K-major UMMA layout).
#include "codec.cuh"
#include "common.cuh"
#include "gemm_raster.cuh"
#include "kernels.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include <mutex>

namespace wv {
namespace {

constexpr int kBM = 128;

template <int KIND> struct GT;
template <> struct GT<kGemmBF16> {
  static constexpr int BN = 256, BK = 64, STAGES = 4, UK = 16, NA = 1, NB = 1, ELEM = 2;
  // output staging: per epilogue warp two slots of 32 rows x 64 bf16 columns
  static constexpr int OUT_STAGE = 4 * 2 * 32 * 128;
  static constexpr uint32_t FMT = 1;
  static constexpr int CODE_BYTES = 0;  // B arrives ready for UMMA
  static constexpr int THREADS = 192;
};
template <> struct GT<kGemmTF32x3> {
  static constexpr int BN = 128, BK = 32, STAGES = 3, UK = 8, NA = 2, NB = 2, ELEM = 4;
  static constexpr uint32_t FMT = 2;
  static constexpr int CODE_BYTES = 0;
  static constexpr int THREADS = 192;
};
// FP8 / NF4 weights: TMA brings the codes (BN x 64 codes) into a staging buffer,
// warps 6.. (8 for FP8, 16 for NF4) write the BF16 tile that UMMA reads.
template <> struct GT<kGemmFP8> {
  static constexpr int BN = 256, BK = 64, STAGES = 3, UK = 16, NA = 1, NB = 1, ELEM = 2;
  static constexpr uint32_t FMT = 1;
  static constexpr int CODE_BYTES = 256 * 64;  // one byte per code
  static constexpr int THREADS = 448;  // 8 dequantisation warps
};
template <> struct GT<kGemmNF4> {
  static constexpr int BN = 256, BK = 64, STAGES = 3, UK = 16, NA = 1, NB = 1, ELEM = 2;
  static constexpr uint32_t FMT = 1;
  static constexpr int CODE_BYTES = 256 * 32;  // two codes per byte
  static constexpr int THREADS = 704;  // 16 dequantisation warps (NF4 conversion is longer)
};
// FormatNone Int8 codes take FP8's layout and warp count; Int4 / FP4 take NF4's.
template <> struct GT<kGemmI8> : GT<kGemmFP8> {};
template <> struct GT<kGemmI4> : GT<kGemmNF4> {};
template <> struct GT<kGemmFP4> : GT<kGemmNF4> {};
template <int KIND> __host__ __device__ constexpr bool byte_codes() { return KIND == kGemmFP8 || KIND == kGemmI8; }
template <int KIND> __host__ __device__ constexpr bool nibble_codes() { return KIND == kGemmNF4 || KIND == kGemmI4 || KIND == kGemmFP4; }
template <int KIND> __host__ __device__ constexpr int out_stage_bytes() { return KIND == kGemmBF16 ? GT<kGemmBF16>::OUT_STAGE : 0; }
// The 16 BF16-exact values a nibble code stands for (before the epilogue scale).
__device__ __forceinline__ float nibble_level(int kind, int c) {
  if (kind == kGemmI4) return (float)(c < 8 ? c : c - 16);                // Int4: two's complement
  if (kind == kGemmFP4) {                                                // FP4 E2M1 (float_codecs.cpp:184)
    const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    return c < 8 ? mag[c] : -mag[c - 8];
  }
  return nf4_level(c);
}

struct KParams {
  int M, N, K, m_tiles, n_tiles, num_tiles, k_blocks;
  int gn;  // N-tiles per raster group (see tile_coords)
  // Split-K (few output tiles, e.g. a decode step's M <= 128 rows): tile t covers
  // k-blocks [sk * kb_per, (sk + 1) * kb_per) of output tile t / ksplit (sk = t %
  // ksplit); its epilogue writes the raw FP32 sums to ws [ksplit, M, N] and
  // splitk_finish_kernel adds the splits in order and applies the epilogue.
  int ksplit, kb_per;
  float* ws;
  void* out;
  int ldo, out_bf16;
  float* out_hi;
  float* out_lo;
  int split_only;  // FP32 output: only out_hi / out_lo are written
  int stage_out;   // plain BF16 output: 64-column groups staged in shared memory, TMA-stored
  const float* b_scale;    // FP8: per-row scales; NF4: per-64 absmax (dequant warps)
  const float* col_scale;  // FP8 only: per-output-column scale applied in the epilogue
  int ldb;
  const float2* rope_tab;
  int rope_cols, head_dim, rope_max_pos;
  const int* positions;
  int pos_mod;
  void* kv_k;
  void* kv_v;
  const int* kv_slot;
  int kv_col0, kv_dim;
  int swiglu, swiglu_cols;
  uint32_t* err;
};

// Bytes of weights in one raster panel (WELVET_B200_GEMM_PANEL_MB, default 24). At
// the QKV shape (K = 4096, 2 MB of BF16 weights per N-tile) 48 MB panels read 2.5x
// the algorithmic bytes from DRAM and 24 MB panels 1.85x, the panel staying in the
// part of the L2 that the A stream leaves it, at equal or slightly shorter times.
inline double panel_bytes() {
  static const double b = [] {
    const char* v = std::getenv("WELVET_B200_GEMM_PANEL_MB");
    const double mb = v && *v ? std::atof(v) : 0.0;
    return (mb > 0.0 ? mb : 24.0) * 1.0e6;
  }();
  return b;
}

// Grouped rasterisation over N: a panel of gn N-tiles of B (the weights: at most
// ~24 MB, chosen on the host) is swept by every M-tile before the next panel, N
// fastest within the panel. The panel stays L2-resident, so B is read from HBM once
// and A once per panel (n_tiles / gn times); the CTAs of one wave share their A
// tiles too. (Grouping 8 M-tiles across all of N instead re-read the whole weight
// matrix once per 8 M-tiles: 3.2x the algorithmic bytes at the QKV shape.)
__device__ __forceinline__ void tile_coords(int t, const KParams& p, int& mb, int& nb) {
  raster_tile(t, p.gn, p.m_tiles, p.n_tiles, mb, nb);
}

// Work of persistent tile index t: output tile (mb, nb) and k-blocks [kb0, kb1).
__device__ __forceinline__ void tile_work(int t, const KParams& p, int& mb, int& nb, int& kb0, int& kb1, int& sk) {
  sk = t % p.ksplit;
  tile_coords(t / p.ksplit, p, mb, nb);
  kb0 = sk * p.kb_per;
  kb1 = min(p.k_blocks, kb0 + p.kb_per);
}

__device__ __forceinline__ void store_vals(const KParams& p, int row, int col, const float* v,
                                           int nvalid) {
  // Decode: K/V columns are scattered into the KV page pools.
  if (p.kv_k && col >= p.kv_col0) {
    int rel = col - p.kv_col0;
    const bool is_v = rel >= p.kv_dim;
    if (is_v) rel -= p.kv_dim;
    const int slot = p.kv_slot[row];
    if (slot < 0) return;
    char* base = static_cast<char*>(is_v ? p.kv_v : p.kv_k);
    // pool layout [page][kv_head][kPageTokens][head_dim]; a 32-column chunk stays
    // inside one head (head_dim is a multiple of 32 on this path)
    const int hd = p.head_dim, nk = p.kv_dim / hd;
    const size_t off = (((size_t)(slot / kPageTokens) * nk + rel / hd) * kPageTokens +
                        slot % kPageTokens) * hd + rel % hd;
    if (p.out_bf16) {
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(base) + off;
      for (int e = 0; e < nvalid; ++e) d[e] = __float2bfloat16_rn(v[e]);
    } else {
      float* d = reinterpret_cast<float*>(base) + off;
      for (int e = 0; e < nvalid; ++e) d[e] = v[e];
    }
    return;
  }
  const size_t off = (size_t)row * p.ldo + col;
  if (p.out_bf16) {
    __nv_bfloat16* d = static_cast<__nv_bfloat16*>(p.out) + off;
    if (nvalid == 32 && (off % 8) == 0) {
#pragma unroll
      for (int e = 0; e < 32; e += 8)
        st_global_v4(d + e, pack_bf16x2(v[e], v[e + 1]), pack_bf16x2(v[e + 2], v[e + 3]),
                     pack_bf16x2(v[e + 4], v[e + 5]), pack_bf16x2(v[e + 6], v[e + 7]));
    } else {
      for (int e = 0; e < nvalid; ++e) d[e] = __float2bfloat16_rn(v[e]);
    }
    return;
  }
  if (!p.split_only) {
    float* d = static_cast<float*>(p.out) + off;
    if (nvalid == 32 && (off % 4) == 0) {
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        st_global_v4(d + e, __float_as_uint(v[e]), __float_as_uint(v[e + 1]),
                     __float_as_uint(v[e + 2]), __float_as_uint(v[e + 3]));
    } else {
      for (int e = 0; e < nvalid; ++e) d[e] = v[e];
    }
  }
  if (p.out_hi) {
    float* h = p.out_hi + off;
    float* l = p.out_lo + off;
    if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(l)) & 15) == 0) {
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float h0 = to_tf32(v[e]), h1 = to_tf32(v[e + 1]), h2 = to_tf32(v[e + 2]), h3 = to_tf32(v[e + 3]);
        st_global_v4(h + e, __float_as_uint(h0), __float_as_uint(h1), __float_as_uint(h2), __float_as_uint(h3));
        st_global_v4(l + e, __float_as_uint(v[e] - h0), __float_as_uint(v[e + 1] - h1),
                     __float_as_uint(v[e + 2] - h2), __float_as_uint(v[e + 3] - h3));
      }
    } else {
      for (int e = 0; e < nvalid; ++e) {
        const float hv = to_tf32(v[e]);
        h[e] = hv;
        l[e] = v[e] - hv;
      }
    }
  }
}

template <int BN>
__device__ __forceinline__ void epilogue_tile(const KParams& p, uint32_t tbase, int row, int n0) {
  const bool row_ok = row < p.M;
  if (p.swiglu) {
    // 32 gate columns then the matching 32 up columns: h = SiLU(gate) * up with
    // SiLU(g) = g / (1 + e^-g), the product rounded once (op_swiglu,
    // shaders/ops_common.metal:27-38)
    for (int c = 0; c < BN && n0 + c < p.N; c += 64) {
      uint32_t g[32], u[32];
      tmem_ld32(tbase + c, g);
      tmem_ld32(tbase + c + 32, u);
      tmem_ld_wait();
      if (row_ok) {
        float h[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float gv = __uint_as_float(g[e]);
          h[e] = __fdiv_rn(gv, 1.f + expf(-gv)) * __uint_as_float(u[e]);
        }
        const int hc = (n0 + c) / 2;
        if (hc < p.swiglu_cols) store_vals(p, row, hc, h, min(32, p.swiglu_cols - hc));
      }
    }
    return;
  }
  const int hd = p.head_dim;
  const bool fuse_rope = p.rope_cols > 0 && (hd == 64 || hd == 128 || hd == 256) && (BN % hd) == 0;
  int pos = 0;
  bool pos_ok = true;
  if (fuse_rope && row_ok) {
    pos = p.positions ? p.positions[row] : (p.pos_mod > 0 ? row % p.pos_mod : row);
    pos_ok = pos >= 0 && pos < p.rope_max_pos;
    if (!pos_ok) atomicCAS(p.err, 0u, 0x100u);
  }
  int c = 0;
  while (c < BN) {
    const int gcol = n0 + c;
    if (gcol >= p.N) break;
    if (fuse_rope && gcol < p.rope_cols) {
      const int half = hd >> 1;
      for (int j = 0; j < half; j += 32) {
        uint32_t x[32], y[32];
        tmem_ld32(tbase + c + j, x);
        tmem_ld32(tbase + c + half + j, y);
        tmem_ld_wait();
        if (row_ok) {
          float xo[32], yo[32];
          const float2* tab = p.rope_tab + (size_t)(pos_ok ? pos : 0) * half + j;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float a = __uint_as_float(x[e]), b = __uint_as_float(y[e]);
            if (p.col_scale) {  // FP8 per-channel scale precedes the rotation
              a *= p.col_scale[gcol + j + e];
              b *= p.col_scale[gcol + half + j + e];
            }
            const float2 cs = pos_ok ? tab[e] : make_float2(1.f, 0.f);
            xo[e] = a * cs.x - b * cs.y;
            yo[e] = a * cs.y + b * cs.x;
          }
          store_vals(p, row, gcol + j, xo, 32);
          store_vals(p, row, gcol + half + j, yo, 32);
        }
      }
      c += hd;
    } else {
      uint32_t x[32];
      tmem_ld32(tbase + c, x);
      tmem_ld_wait();
      if (row_ok) {
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(x[e]);
        if (p.col_scale) {  // FP8: per-output-channel scale factors out of the K sum
          for (int e = 0; e < 32 && gcol + e < p.N; ++e) v[e] *= p.col_scale[gcol + e];
        }
        store_vals(p, row, gcol, v, min(32, p.N - gcol));
      }
      c += 32;
    }
  }
}

// Split-K epilogue: the tile's raw FP32 sums into the split's slice of ws.
template <int BN>
__device__ __forceinline__ void epilogue_partial(const KParams& p, uint32_t tbase, int row, int n0, int sk) {
  const bool row_ok = row < p.M;
  float* dst = p.ws + ((size_t)sk * p.M + (row_ok ? row : 0)) * p.N;
  for (int c = 0; c < BN && n0 + c < p.N; c += 32) {
    uint32_t x[32];
    tmem_ld32(tbase + c, x);
    tmem_ld_wait();
    if (!row_ok) continue;
    const int gcol = n0 + c;
    if (gcol + 32 <= p.N && (((size_t)sk * p.M + row) * p.N + gcol) % 4 == 0) {
#pragma unroll
      for (int e = 0; e < 32; e += 4) st_global_v4(dst + gcol + e, x[e], x[e + 1], x[e + 2], x[e + 3]);
    } else {
      for (int e = 0; e < 32 && gcol + e < p.N; ++e) dst[gcol + e] = __uint_as_float(x[e]);
    }
  }
}

// Sum of the split-K partials of (row, col), in split order.
__device__ __forceinline__ float splitk_sum(const KParams& p, int row, int col) {
  float v = 0.f;
  for (int s_ = 0; s_ < p.ksplit; ++s_) v += __ldg(p.ws + ((size_t)s_ * p.M + row) * p.N + col);
  if (p.col_scale) v *= p.col_scale[col];
  return v;
}

// The epilogue of split-K GEMMs (per-row scale, RoPE on the first rope_cols
// columns, output type), one output element per thread; a RoPE element reads its
// pair partner's sums too. RoPE is applied where epilogue_tile<BN> would fuse it.
template <int BN>
__global__ void splitk_finish_kernel(const KParams p) {
  const int hd = p.head_dim;
  const bool fuse_rope = p.rope_cols > 0 && (hd == 64 || hd == 128 || hd == 256) && (BN % hd) == 0;
  const int64_t total = (int64_t)p.M * p.N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / p.N), col = (int)(i % p.N);
    float v = splitk_sum(p, row, col);
    if (fuse_rope && col < p.rope_cols) {
      const int half = hd >> 1, in_head = col % hd;
      const int pos = p.positions ? p.positions[row] : (p.pos_mod > 0 ? row % p.pos_mod : row);
      const bool pos_ok = pos >= 0 && pos < p.rope_max_pos;
      if (!pos_ok) atomicCAS(p.err, 0u, 0x100u);
      const float2 cs = pos_ok ? p.rope_tab[(size_t)pos * half + (in_head % half)] : make_float2(1.f, 0.f);
      if (in_head < half) {
        const float b = splitk_sum(p, row, col + half);
        v = v * cs.x - b * cs.y;
      } else {
        const float a = splitk_sum(p, row, col - half);
        v = a * cs.y + v * cs.x;
      }
    }
    const size_t off = (size_t)row * p.ldo + col;
    if (p.out_bf16) static_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(v);
    else static_cast<float*>(p.out)[off] = v;
  }
}

// Plain BF16 output through shared memory: the 32 rows of this warp (TMEM lanes)
// are written in 64-column groups, each staged as [32 rows][128 B] in the 128-byte
// swizzle (slot n_staged & 1 of the warp's two) and stored by one TMA store, so the
// output leaves in whole 128-byte lines instead of one 16-byte piece of 32 rows per
// store instruction; TMA clips rows past M and columns past N. Before a slot is
// rewritten, lane 0 waits until at most one earlier store is still reading.
template <int BN>
__device__ __forceinline__ void epilogue_staged(const KParams& p, uint32_t tbase, const CUtensorMap* tmO,
                                                uint8_t* stage, int row0, int n0, int lane, int& n_staged) {
  for (int g = 0; g < BN / 64; ++g) {
    const int gcol = n0 + 64 * g;
    if (gcol >= p.N) break;
    uint32_t x0[32], x1[32];
    tmem_ld32(tbase + 64 * g, x0);
    tmem_ld32(tbase + 64 * g + 32, x1);
    tmem_ld_wait();
    uint32_t pk[32];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      pk[e] = pack_bf16x2(__uint_as_float(x0[2 * e]), __uint_as_float(x0[2 * e + 1]));
      pk[16 + e] = pack_bf16x2(__uint_as_float(x1[2 * e]), __uint_as_float(x1[2 * e + 1]));
    }
    uint8_t* buf = stage + (n_staged & 1) * 4096;
    if (lane == 0) bulk_wait_read1();
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 8; ++c)
      st_shared_v4(buf + lane * 128 + ((c ^ (lane & 7)) << 4), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmO, buf, gcol, row0);
      bulk_commit();
    }
    ++n_staged;
  }
}

// 16 bytes of a 128-byte-swizzled K-major row: chunk index XOR (row mod 8).
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk16) {
  return (uint32_t)(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

template <int KIND>
__global__ void __launch_bounds__(GT<KIND>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmB2,
                   const __grid_constant__ CUtensorMap tmO, const KParams p) {
  using T = GT<KIND>;
  constexpr int BN = T::BN, BK = T::BK, S = T::STAGES;
  constexpr int A_BYTES = kBM * BK * T::ELEM;
  constexpr int B_BYTES = BN * BK * T::ELEM;
  constexpr bool XFORM = T::CODE_BYTES > 0;
  constexpr int STAGE_BYTES = T::NA * A_BYTES + T::NB * B_BYTES + T::CODE_BYTES;
  constexpr uint32_t IDESC = idesc_make(T::FMT, kBM, BN, 0, 0);
  constexpr uint32_t TMEM_COLS = 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int OUT_STAGE = out_stage_bytes<KIND>();
  uint8_t* out_stage = smem + S * STAGE_BYTES;  // [warp][slot][32 rows][128 B], 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * STAGE_BYTES + OUT_STAGE);
  uint64_t* empty = full + S;
  uint64_t* xfull = empty + S;  // dequantised B ready (FP8/NF4)
  uint64_t* accf = xfull + S;
  uint64_t* acce = accf + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = (int)warp_id(), lane = (int)lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&xfull[s], T::THREADS - 192);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        int mb, nb, kb0, kb1, sk;
        tile_work(t, p, mb, nb, kb0, kb1, sk);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, kErrWaitEmpty)) goto done;
          uint8_t* sb = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES - (XFORM ? B_BYTES : 0));
          tma_load_2d(sb, &tmA, &full[stage], kb * BK, mb * kBM);
          if constexpr (T::NA == 2) tma_load_2d(sb + A_BYTES, &tmA2, &full[stage], kb * BK, mb * kBM);
          if constexpr (XFORM) {
            // Codes for (BN rows) x (64 k): fp8 64 bytes/row, nf4 32 bytes/row.
            constexpr int kx = byte_codes<KIND>() ? BK : BK / 2;
            tma_load_2d(sb + T::NA * A_BYTES + B_BYTES, &tmB, &full[stage], kb * kx, nb * BN);
          } else {
            tma_load_2d(sb + T::NA * A_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
            if constexpr (T::NB == 2)
              tma_load_2d(sb + T::NA * A_BYTES + B_BYTES, &tmB2, &full[stage], kb * BK, nb * BN);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- UMMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        if (!mbar_wait(&acce[acc], acc_phase ^ 1, abort_flag, p.err, kErrWaitAccEmpty)) goto done;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        int mb, nb, kb0, kb1, sk;
        tile_work(t, p, mb, nb, kb0, kb1, sk);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrWaitFull)) goto done;
          if constexpr (XFORM) {
            if (!mbar_wait(&xfull[stage], phase, abort_flag, p.err, kErrWaitFull)) goto done;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t a1 = a0 + A_BYTES;
          const uint32_t b0 = a0 + T::NA * A_BYTES;
          const uint32_t b1 = b0 + B_BYTES;
#pragma unroll
          for (int ks = 0; ks < BK / T::UK; ++ks) {
            const uint32_t off = (uint32_t)(ks * T::UK * T::ELEM);
            const uint64_t ad = sdesc_sw128(a0 + off, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + off, 16, 1024);
            const uint32_t accum = (kb != kb0 || ks != 0) ? 1u : 0u;
            if constexpr (KIND == kGemmTF32x3) {
              umma_tf32_ss(d, sdesc_sw128(a1 + off, 16, 1024), bd, IDESC, accum);
              umma_tf32_ss(d, ad, sdesc_sw128(b1 + off, 16, 1024), IDESC, 1);
              umma_tf32_ss(d, ad, bd, IDESC, 1);
            } else {
              umma_f16_ss(d, ad, bd, IDESC, accum);
            }
          }
          umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&accf[acc]);
        acc ^= 1;
        if (!acc) acc_phase ^= 1;
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    int n_staged = 0;  // 64-column groups this warp has staged (slot = n_staged & 1)
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mb, nb, kb0, kb1, sk;
      tile_work(t, p, mb, nb, kb0, kb1, sk);
      bool ok = mbar_wait(&accf[acc], acc_phase, abort_flag, p.err, kErrWaitAccFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN);
      if (p.ksplit > 1) epilogue_partial<BN>(p, tbase, mb * kBM + 32 * q + lane, nb * BN, sk);
      else if (OUT_STAGE > 0 && p.stage_out)
        epilogue_staged<BN>(p, tbase, &tmO, out_stage + q * 8192, mb * kBM + 32 * q, nb * BN, lane, n_staged);
      else epilogue_tile<BN>(p, tbase, mb * kBM + 32 * q + lane, nb * BN);
      tc_fence_before();
      mbar_arrive(&acce[acc]);
      acc ^= 1;
      if (!acc) acc_phase ^= 1;
    }
  } else if constexpr (XFORM) {
    // --------------------------------------------- B dequantisation (FP8/NF4)
    // XT threads; thread xt writes 16-byte (8 x bf16) chunk ch = xt % 8 of
    // rows xt / 8 + RS j (j < BN / RS, RS = XT / 8) of the swizzled tile. Each
    // warp's conversions are dependent chains per row, so more warps (not more
    // rows per warp) keep the conversion pipes busy.
    constexpr int XT = T::THREADS - 192, RS = XT / 8;
    const int xt = threadIdx.x - 192;
    const int ch = xt & 7, r0 = xt >> 3;
    constexpr int RPT = BN / RS;  // rows per thread
    // NF4: the 16 levels as BF16, held in registers as two byte planes (low and
    // high bytes, four levels per register), so a level lookup is a byte permute
    // instead of a shared-memory load.
    uint32_t lvl_lo[4] = {0, 0, 0, 0}, lvl_hi[4] = {0, 0, 0, 0};
    if constexpr (nibble_codes<KIND>()) {
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t h = pack_bf16x2(nibble_level(KIND, c), 0.f) & 0xffffu;
        lvl_lo[c >> 2] |= (h & 0xffu) << (8 * (c & 3));
        lvl_hi[c >> 2] |= (h >> 8) << (8 * (c & 3));
      }
    }
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mb, nb, kb0, kb1, sk;
      tile_work(t, p, mb, nb, kb0, kb1, sk);
      for (int kb = kb0; kb < kb1; ++kb) {
        // NF4: the 64-code block of this k-block has one absmax per row; the loads
        // are issued before the wait so their latency hides behind it.
        float amax[KIND == kGemmNF4 ? RPT : 1];
        if constexpr (KIND == kGemmNF4) {
#pragma unroll
          for (int j = 0; j < RPT; ++j) {
            const int n = nb * BN + r0 + RS * j;
            amax[j] = n < p.N ? __ldg(p.b_scale + (size_t)n * (p.K / 64) + kb) : 0.f;
          }
        }
        bool ok = mbar_wait(&full[stage], phase, abort_flag, p.err, kErrWaitFull);
        if (!__all_sync(0xffffffffu, ok)) goto done;
        uint8_t* sb = smem + stage * STAGE_BYTES;
        uint8_t* btile = sb + T::NA * A_BYTES;
        const uint8_t* codes = btile + B_BYTES;
        // All codes of this thread's rows are loaded before any converted chunk is
        // stored: the stores may alias the loads as far as the compiler knows, so
        // interleaving them would serialise every row on the shared-memory latency.
        using CodeT = typename std::conditional<byte_codes<KIND>(), uint2, uint32_t>::type;
        CodeT cw[RPT];
#pragma unroll
        for (int j = 0; j < RPT; ++j)
          cw[j] = *reinterpret_cast<const CodeT*>(codes + (r0 + RS * j) * (byte_codes<KIND>() ? 64 : 32) +
                                                  ch * (byte_codes<KIND>() ? 8 : 4));
        // Converted chunks are held in registers and stored after the last
        // conversion: both conversions are register-only (no shared-memory loads),
        // so the stores leave as one burst.
        uint32_t w[RPT][4];
#pragma unroll
        for (int j = 0; j < RPT; ++j) {  // fully unrolled: cw[], amax[], w[] stay in registers
          if constexpr (KIND == kGemmFP8) {
            // Codes are normalised E4M3 (no subnormal codes, no 0x7f/0xff: the
            // mount maps them to the values the reference decoder gives, +-0 and
            // +-448), so the hardware E4M3 -> F16 conversion is exact, as is F16 ->
            // F32 -> BF16 for these 4-bit-mantissa values.
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t word = e < 2 ? cw[j].x : cw[j].y;
              const uint16_t pair = (uint16_t)(word >> ((e & 1) * 16));
              uint32_t h2;
              float lo, hi;
              asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(pair));
              asm("{.reg .f16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.f32.f16 %0, a;\n\tcvt.f32.f16 %1, b;\n\t}"
                  : "=f"(lo), "=f"(hi) : "r"(h2));
              w[j][e] = pack_bf16x2(lo, hi);
            }
          } else if constexpr (KIND == kGemmI8) {
            // Int8 codes are exact in BF16: each byte becomes the float 2^23 + (b ^
            // 0x80) by a byte permute under the exponent of 2^23, minus 2^23 + 128
            // (one packed f32x2 add per pair), then one RN pack (exact) per pair.
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t word = (e < 2 ? cw[j].x : cw[j].y) ^ 0x80808080u;
              const int b0 = 2 * (e & 1);
              const float lo = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u + b0)) - 8388736.0f;
              const float hi = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7541u + b0)) - 8388736.0f;
              w[j][e] = pack_bf16x2(lo, hi);
            }
          } else {
            // Nibble k of the code word is element k (low nibble first). Each
            // nibble's low three bits select a byte from a register pair (levels
            // 0-7 or 8-15; __byte_perm reads three bits per selector nibble and
            // the low 16 bits of the selector). A second permute picks, per byte,
            // the pair that bit 3 names (selector nibble j + 4 * bit3). The two
            // planes are then interleaved into BF16 pairs and scaled by the block
            // absmax with one BF16x2 multiply: bf16(bf16(level) * bf16(absmax)).
            const __nv_bfloat162 am2 = __float2bfloat162_rn(KIND == kGemmNF4 ? amax[j] : 1.f);
            const uint32_t code = cw[j];
            const uint32_t pick = ((code >> 1) & 0x44444444u) | 0x32103210u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t s4 = code >> (16 * h), p4 = pick >> (16 * h);
              const uint32_t lo = __byte_perm(__byte_perm(lvl_lo[0], lvl_lo[1], s4),
                                              __byte_perm(lvl_lo[2], lvl_lo[3], s4), p4);
              const uint32_t hi = __byte_perm(__byte_perm(lvl_hi[0], lvl_hi[1], s4),
                                              __byte_perm(lvl_hi[2], lvl_hi[3], s4), p4);
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                uint32_t v = __byte_perm(lo, hi, q ? 0x7362u : 0x5140u);
                if constexpr (KIND == kGemmNF4) {
                  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&v), am2);
                  v = *reinterpret_cast<uint32_t*>(&r);
                }
                w[j][2 * h + q] = v;
              }
            }
          }
        }
#pragma unroll
        for (int j = 0; j < RPT; ++j)
          *reinterpret_cast<uint4*>(btile + sw128_offset(r0 + RS * j, ch)) =
              make_uint4(w[j][0], w[j][1], w[j][2], w[j][3]);
        fence_proxy_async_smem();
        mbar_arrive(&xfull[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }
done:
  // the staged output stores of each epilogue warp are complete (they read shared
  // memory until then)
  if (OUT_STAGE > 0 && warp >= 2 && warp < 6 && lane == 0) bulk_wait0();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

} // namespace

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool make_map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t ld_elems, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tma_2d(void* map128, const void* base, int dt, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t ld_elems, uint32_t box_inner, uint32_t box_outer, int sw) {
  return make_map_2d(static_cast<CUtensorMap*>(map128), base, static_cast<CUtensorMapDataType>(dt),
                     elem_bytes, inner, outer, ld_elems, box_inner, box_outer,
                     static_cast<CUtensorMapSwizzle>(sw));
}

namespace {

// Split-K factor of a GEMM: when its output tiles fill under half of the SMs (a
// decode step's few rows), the K range is split so that about one tile per SM runs;
// needs the caller's FP32 workspace (splitk_ws, ksplit * M * N floats) and the plain
// epilogue (no SwiGLU, KV scatter or TF32 output split).
// (query: the factor an unlimited workspace would allow).
int splitk_count(const GemmArgs& g, int spatial, int k_blocks, int* kb_per, bool query = false) {
  *kb_per = k_blocks;
  if ((!g.splitk_ws && !query) || g.swiglu || g.kv_k || g.out_hi || spatial * 2 > g.sm_count || k_blocks < 2)
    return 1;
  const int want = std::max(1, g.sm_count / spatial);
  int per = (k_blocks + want - 1) / want;
  int ks = (k_blocks + per - 1) / per;
  while (!query && ks > 1 && (size_t)ks * g.M * g.N > g.splitk_ws_floats) {  // fit the workspace
    ++per;
    ks = (k_blocks + per - 1) / per;
  }
  *kb_per = ks > 1 ? per : k_blocks;
  return ks;
}

template <int KIND> size_t smem_bytes() {
  using T = GT<KIND>;
  const size_t stage = T::NA * kBM * T::BK * T::ELEM + T::NB * T::BN * T::BK * T::ELEM + T::CODE_BYTES;
  return 1024 + T::STAGES * stage + out_stage_bytes<KIND>() + 8 * (3 * T::STAGES + 4) + 16 + 512;
}

template <int KIND> cudaError_t launch(const GemmArgs& g, cudaStream_t stream) {
  using T = GT<KIND>;
  CUtensorMap ta{}, ta2{}, tb{}, tb2{};
  const bool f32 = KIND == kGemmTF32x3;
  const CUtensorMapDataType adt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int ae = f32 ? 4 : 2;
  if (!make_map_2d(&ta, g.a, adt, ae, g.K, g.M, g.lda, T::BK, kBM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  ta2 = ta;
  if (f32 && !make_map_2d(&ta2, g.a_lo, adt, ae, g.K, g.M, g.lda, T::BK, kBM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (byte_codes<KIND>()) {
    if (!make_map_2d(&tb, g.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, g.N, g.ldb, 64, T::BN,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else if (nibble_codes<KIND>()) {
    if (!make_map_2d(&tb, g.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K / 2, g.N, g.ldb / 2, 32, T::BN,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    if (!make_map_2d(&tb, g.b, adt, ae, g.K, g.N, g.ldb, T::BK, T::BN, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  tb2 = tb;
  if (f32 && !make_map_2d(&tb2, g.b_lo, adt, ae, g.K, g.N, g.ldb, T::BK, T::BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;

  KParams p{};
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.m_tiles = (g.M + kBM - 1) / kBM;
  p.n_tiles = (g.N + T::BN - 1) / T::BN;
  p.k_blocks = (g.K + T::BK - 1) / T::BK;
  p.ksplit = splitk_count(g, p.m_tiles * p.n_tiles, p.k_blocks, &p.kb_per);
  p.ws = p.ksplit > 1 ? g.splitk_ws : nullptr;
  p.num_tiles = p.m_tiles * p.n_tiles * p.ksplit;
  {
    // B bytes of one N-tile as stored in HBM (codes for FP8 / NF4, both TF32 parts)
    const double b_elem = byte_codes<KIND>() ? 1.0 : nibble_codes<KIND>() ? 0.5 : (double)(T::ELEM * T::NB);
    const double panel = (double)T::BN * g.K * b_elem;
    const int gn = (int)std::max(1.0, std::floor(panel_bytes() / std::max(panel, 1.0)));
    p.gn = std::min(p.n_tiles, gn);
  }
  p.out = g.out;
  p.ldo = g.ldo;
  p.out_bf16 = g.out_bf16;
  p.out_hi = g.out_hi;
  p.out_lo = g.out_lo;
  p.split_only = g.split_only && g.out_hi ? 1 : 0;
  p.b_scale = g.b_scale;
  p.ldb = g.ldb;
  p.col_scale = (KIND == kGemmFP8 || KIND == kGemmI8 || KIND == kGemmI4 || KIND == kGemmFP4) ? g.b_scale : nullptr;
  p.rope_tab = g.rope_tab;
  p.rope_cols = g.rope_tab ? g.rope_cols : 0;
  p.head_dim = g.head_dim;
  p.rope_max_pos = g.rope_max_pos;
  p.positions = g.positions;
  p.pos_mod = g.pos_mod;
  p.kv_k = g.kv_k;
  p.kv_v = g.kv_v;
  p.kv_slot = g.kv_slot;
  p.kv_col0 = g.kv_col0;
  p.kv_dim = g.kv_dim;
  p.swiglu = g.swiglu;
  p.swiglu_cols = g.swiglu_cols > 0 ? g.swiglu_cols : g.N / 2;
  p.err = g.err;

  // Plain BF16 output (no split, RoPE, KV scatter, SwiGLU or TF32 split): staged
  // 64-column groups stored by TMA ([rows][ldo], boxes of 64 columns x 32 rows).
  CUtensorMap to = ta;
  p.stage_out = 0;
  if (out_stage_bytes<KIND>() > 0 && g.out_bf16 && p.ksplit == 1 && !g.swiglu && !g.kv_k && !g.out_hi &&
      p.rope_cols == 0 && (reinterpret_cast<uintptr_t>(g.out) & 15) == 0 && ((size_t)g.ldo * 2) % 16 == 0 &&
      make_map_2d(&to, g.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.N, g.M, g.ldo, 64, 32,
                  CU_TENSOR_MAP_SWIZZLE_128B))
    p.stage_out = 1;
  const size_t smem = smem_bytes<KIND>();
  static cudaError_t attr = cudaFuncSetAttribute(gemm_tc_kernel<KIND>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (attr != cudaSuccess) return attr;
  const int grid = std::max(1, std::min(p.num_tiles, g.sm_count));
  gemm_tc_kernel<KIND><<<grid, T::THREADS, smem, stream>>>(ta, ta2, tb, tb2, to, p);
  if (p.ksplit > 1) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t total = (int64_t)g.M * g.N;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)g.sm_count * 8);
    splitk_finish_kernel<T::BN><<<blocks, 256, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

} // namespace

bool gemm_tc_supported(const GemmArgs& g) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return false;
  const int ae = g.kind == kGemmTF32x3 ? 4 : 2;
  // TMA: 16-byte aligned bases and row strides.
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(g.a) || ((size_t)g.lda * ae) % 16) return false;
  if (g.kind == kGemmTF32x3 && (!al16(g.a_lo) || !al16(g.b_lo))) return false;
  if (!al16(g.b)) return false;
  const bool bytes = g.kind == kGemmFP8 || g.kind == kGemmI8;
  const bool nibbles = g.kind == kGemmNF4 || g.kind == kGemmI4 || g.kind == kGemmFP4;
  if (g.kind < kGemmBF16 || g.kind > kGemmFP4) return false;
  if (bytes || nibbles) {
    if (g.K % 64) return false;
    if (bytes && g.ldb % 16) return false;
    if (nibbles && (g.ldb / 2) % 16) return false;
    if (g.kind != kGemmFP4 && !g.b_scale) return false;
  } else if (((size_t)g.ldb * ae) % 16) {
    return false;
  }
  if (g.kv_k && (g.kv_dim % 32 || g.kv_col0 % 32 || g.head_dim % 32)) return false;
  if (g.swiglu && (g.N % 64 || g.rope_cols || g.kv_k || (g.kind != kGemmBF16 && g.kind != kGemmTF32x3))) return false;
  return encode_fn() != nullptr;
}

namespace {
int splitk_of(const GemmArgs& g, bool query) {
  const int bn = g.kind == kGemmTF32x3 ? GT<kGemmTF32x3>::BN : GT<kGemmBF16>::BN;
  const int bk = g.kind == kGemmTF32x3 ? GT<kGemmTF32x3>::BK : GT<kGemmBF16>::BK;
  int kb_per = 0;
  const int spatial = ((g.M + kBM - 1) / kBM) * ((g.N + bn - 1) / bn);
  return splitk_count(g, spatial, (g.K + bk - 1) / bk, &kb_per, query);
}
}  // namespace

size_t gemm_tc_splitk_floats(const GemmArgs& g) {
  const int ks = splitk_of(g, true);
  return ks > 1 ? (size_t)ks * g.M * g.N : 0;
}

int gemm_tc_launches(const GemmArgs& g) { return splitk_of(g, false) > 1 ? 2 : 1; }

cudaError_t gemm_tc(const GemmArgs& g, cudaStream_t stream) {
  if (!gemm_tc_supported(g)) return cudaErrorInvalidValue;
  switch (g.kind) {
  case kGemmBF16: return launch<kGemmBF16>(g, stream);
  case kGemmTF32x3: return launch<kGemmTF32x3>(g, stream);
  case kGemmFP8: return launch<kGemmFP8>(g, stream);
  case kGemmNF4: return launch<kGemmNF4>(g, stream);
  case kGemmI8: return launch<kGemmI8>(g, stream);
  case kGemmI4: return launch<kGemmI4>(g, stream);
  case kGemmFP4: return launch<kGemmFP4>(g, stream);
  default: return cudaErrorInvalidValue;
  }
}

} // namespace wv
