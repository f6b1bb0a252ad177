// Few-row BF16 projection of a decode step: out = x W^T for M <= 64 rows (one new
// token per sequence), the Dense forward of the reference's decode path
// (shaders/welvet_dense.metal:54-85 per output, src/layers/mha/mha.cpp:138-205 for
// the q/k/v and output projections), written for what bounds it on the B200: the
// weight matrix is read from HBM once, and at these sizes (a few to a hundred MB)
// the time is one memory round trip plus the transfer, so every load is issued up
// front and the M rows ride along on m16n8k16 tensor-core MMAs.
//
// Work split (weights as the A operand, "swap AB"): a CTA owns 128 output columns
// (128 weight rows = the M = 128 rows of a tcgen05 MMA) over a 512-wide K slice
// (256 or 128 wide when that keeps the grid in one wave with more CTAs), the batch
// rows are the MMA's N (a multiple of 16, zero-filled past M by TMA); a
// thread-block cluster of ks = K / slice CTAs (at most 8) along K covers the whole K
// range. A TMA thread loads the slice's 64-wide k blocks of W (16 KB each) and x —
// all at once when the grid is one wave (one CTA per SM), else through a
// three-stage ring (two CTAs per SM) — one thread issues 4 UMMAs (K = 16) per block
// into a TMEM accumulator [128 lanes = output columns][N columns = batch rows], and
// four warps read it back. Each weight byte crosses shared memory once (an mma.sync
// form re-read the x fragments once per 8 output columns: ~1 MB of shared-memory
// traffic per CTA, 10 us of a 15 us kernel).
//
// Epilogue: each CTA copies the FP32 partial of batch rows [r R, (r+1) R) into CTA
// r's inbox (16-byte distributed shared memory stores); after one cluster barrier
// CTA r sums its inbox in cluster-rank order (deterministic) and applies RoPE (rotate-half pairs inside a head: a head
// lies inside one 128-column tile for head_dim 32/64/128), then stores bf16 rows,
// with the K and V column ranges scattered into the KV page pools (the cache
// append) when kv_k is given.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace wv {
namespace {

constexpr int kThreads = 192;    // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kNC = 128;         // output columns per CTA (the MMA's M)
constexpr int kSlice = 512;      // K per CTA
constexpr int kBK = 64;          // k per block (one 128-byte swizzled row)
constexpr int kBlocks = kSlice / kBK;
constexpr int kNBMax = 64;       // batch rows (MMA N) at most
constexpr int kWBytes = kNC * kBK * 2;      // 16 KB
constexpr int kXBytes = kNBMax * kBK * 2;   // 8 KB
constexpr int kStageBytes = kWBytes + kXBytes;
constexpr int kRedLd = kNC;     // row of a partial tile (floats)
constexpr int kMaxCluster = 8;
// S stages: all eight k blocks of the slice in flight at once (S = 8, one CTA per SM,
// for grids of one wave) or a three-stage ring (two CTAs per SM). IR: rows of the
// inbox, ks x ceil(nb / ks) (64 when ks divides nb, at most 71).
template <int S, int IR> constexpr int smem_bytes() { return 1024 + S * kStageBytes + IR * kRedLd * 4 + 256; }
static_assert(smem_bytes<8, kNBMax>() <= 227 * 1024, "shared memory");
static_assert(2 * smem_bytes<3, kNBMax + kMaxCluster>() <= 228 * 1024, "two CTAs per SM");
static_assert(2 * kNBMax * kRedLd * 4 <= 3 * kStageBytes, "partial and summed rows fit in the ring");

struct VParams {
  int M, N, K, ks, nb;  // nb: batch rows rounded up to 16 (the MMA's N)
  int kb;               // 64-wide k blocks per CTA (the K slice is kb * 64)
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

__device__ __forceinline__ void st_dsmem_v4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}

template <int S, int IR>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_decode_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                       const VParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // inbox [source rank][row of this CTA's slice][kRedLd]: the cluster's partial sums
  // of this CTA's rows, written by every CTA of the cluster (itself included)
  float* inbox = reinterpret_cast<float*>(smem + S * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kStageBytes + IR * kRedLd * 4);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int ks = p.ks;
  const int rank = ks > 1 ? (int)cluster_rank() : 0;
  const int tile = blockIdx.x / ks;
  const int n0 = tile * kNC;
  const int kbeg = rank * p.kb * kBK;
  const int warp = (int)warp_id(), lane = (int)lane_id(), tid = (int)threadIdx.x;
  const int rpr = (p.nb + ks - 1) / ks;  // batch rows per CTA of the cluster

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kNBMax);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // everything but the weight loads reads or writes what the previous kernel may
  // still be producing or reading
  if (warp != 0) pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      const uint32_t bytes = (uint32_t)(kWBytes + p.nb * kBK * 2);
      // The weights do not depend on the previous kernel: the first S blocks of W
      // are requested before waiting for it (programmatic dependent launch), x after.
      const int first = min(S, p.kb);
      for (int b = 0; b < first; ++b) {
        mbar_arrive_expect_tx(&full[b], bytes);
        tma_load_2d(smem + b * kStageBytes, &tmW, &full[b], kbeg + b * kBK, n0);
      }
      pdl_wait();
      for (int b = 0; b < first; ++b)
        tma_load_2d(smem + b * kStageBytes + kWBytes, &tmX, &full[b], kbeg + b * kBK, 0);
      for (int b = S; b < p.kb; ++b) {
        const int s = b % S;
        if (!mbar_wait(&empty[s], ((b / S) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        uint8_t* st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_2d(st, &tmW, &full[s], kbeg + b * kBK, n0);
        tma_load_2d(st + kWBytes, &tmX, &full[s], kbeg + b * kBK, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_make(1, kNC, p.nb, 0, 0);
      for (int b = 0; b < p.kb; ++b) {
        const int s = b % S;
        if (!mbar_wait(&full[s], (b / S) & 1, abort_flag, p.err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t wa = smem_u32(smem + s * kStageBytes), xa = wa + kWBytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16_ss(tmem, sdesc_sw128(wa + 32 * kk, 16, 1024), sdesc_sw128(xa + 32 * kk, 16, 1024), idesc,
                      (b > 0 || kk > 0) ? 1u : 0u);
        if (S < p.kb) umma_commit(&empty[s]);
      }
      umma_commit(acc_full);
    }
  }
  // ---------------------------------- accumulator -> the row owners' inboxes
  // (warps 2-5: TMEM lane quadrant warp % 4 = output columns, columns = batch rows)
  // The tile goes to shared memory first (red, over the ring: this CTA's MMAs are
  // complete and no other CTA writes the ring), then every thread copies 16-byte
  // pieces of its rows to their owners: batch row b belongs to cluster rank b / rpr,
  // which receives it in inbox[rank].
  float* red = reinterpret_cast<float*>(smem);  // [nb][kRedLd]
  bool ok = true;
  if (warp >= 2) {
    ok = mbar_wait(acc_full, 0, abort_flag, p.err, kErrWaitAccFull);
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const int qd = warp & 3, col = 32 * qd + lane;
      for (int c0 = 0; c0 < p.nb; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * qd) << 16) + (uint32_t)c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c0 + e < p.nb) red[(c0 + e) * kRedLd + col] = __uint_as_float(v[e]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kNBMax);
  }
  for (int i = tid; i < p.nb * (kRedLd / 4); i += kThreads) {
    const int b = i / (kRedLd / 4), c4 = i % (kRedLd / 4);
    const int q = b / rpr, lr = b - q * rpr;
    const float4 v = reinterpret_cast<const float4*>(red + b * kRedLd)[c4];
    float4* dst = reinterpret_cast<float4*>(inbox + (rank * rpr + lr) * kRedLd) + c4;
    if (ks > 1) st_dsmem_v4(dsmem_addr(dst, (uint32_t)q), v);
    else *dst = v;
  }
  if (ks > 1) cluster_sync();  // every CTA's rows are in their owners' inboxes
  else __syncthreads();
  // Rows of this CTA's slice summed in rank order into fin (the ring is free: this
  // CTA's MMAs are complete, and no other CTA writes it). Epilogue thread t handles
  // columns [4 (t % 32), + 4) of local rows t / 32 + 4 it.
  float* fin = red + kNBMax * kRedLd;  // [rpr][kRedLd] (after red in the ring)
  const int t = tid - 64;
  const int col = 4 * (t & 31), rsub = t >> 5;
  const int r0 = rank * rpr, r1 = min(p.nb, r0 + rpr);
  if (t >= 0) {
    for (int lr = rsub; lr < r1 - r0; lr += 4) {
      float4 sm = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < ks; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(inbox + (q * rpr + lr) * kRedLd + col);
        sm.x += v.x;
        sm.y += v.y;
        sm.z += v.z;
        sm.w += v.w;
      }
      *reinterpret_cast<float4*>(fin + lr * kRedLd + col) = sm;
    }
  }
  __syncthreads();
  if (t < 0 || !ok) return;
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
  for (int lr = rsub; lr < min(r1, p.M) - r0; lr += 4) {
    const int row = r0 + lr;
    float4 v = *reinterpret_cast<const float4*>(fin + lr * kRedLd + col);
    if (roped) {
      const int pos = p.positions ? p.positions[row] : (p.pos_mod > 0 ? row % p.pos_mod : row);
      const bool pos_ok = pos >= 0 && pos < p.rope_max_pos;
      if (!pos_ok) atomicCAS(p.err, 0u, 0x100u);
      const float4 o = *reinterpret_cast<const float4*>(fin + lr * kRedLd + pcol);
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

template <int S, int IR>
cudaError_t launch(const CUtensorMap* maps, const VParams& p, int tiles, cudaStream_t s) {
  auto kern = gemv_decode_kernel<S, IR>;
  static const cudaError_t ready = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                        smem_bytes<S, IR>());
  if (ready != cudaSuccess) return ready;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(tiles * p.ks, 1, 1);
  lc.blockDim = dim3(kThreads, 1, 1);
  lc.dynamicSmemBytes = smem_bytes<S, IR>();
  lc.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = p.ks;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait above
  at[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = at;
  lc.numAttrs = 2;
  return cudaLaunchKernelEx(&lc, kern, maps[0], maps[1], p);
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
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.nb = (a.M + 15) / 16 * 16;
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
  // K slices of 512 (eight k blocks) per CTA; halved (down to 128) while the
  // cluster stays at 4 CTAs or fewer and the grid within one wave, so that short-K
  // projections (a head shard's output projection: K = 512, 32 CTAs -> 128) spread
  // their weight stream over more SMs. Larger clusters lost more in the distributed
  // shared-memory reduction than they gained (K = 2048 at 8 CTAs: 12.7 -> 18.8 us).
  int slice = kSlice;
  while (slice > 2 * kBK && a.K % (slice / 2) == 0 && a.K / (slice / 2) <= 4 &&
         tiles * (a.K / (slice / 2)) <= a.sm_count && p.nb % (a.K / (slice / 2)) == 0)
    slice /= 2;
  p.ks = a.K / slice;
  p.kb = slice / kBK;
  alignas(64) CUtensorMap maps[2];
  const int BF16 = (int)CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, SW = (int)CU_TENSOR_MAP_SWIZZLE_128B;
  // W [N rows][K]: 128-row boxes; x [M rows][K]: boxes of nb rows, rows past M
  // zero-filled
  if (!make_tma_2d(&maps[0], a.b, BF16, 2, a.K, a.N, a.ldb, kBK, kNC, SW) ||
      !make_tma_2d(&maps[1], a.a, BF16, 2, a.K, a.M, a.lda, kBK, p.nb, SW))
    return cudaErrorInvalidValue;
  // one wave (and a cluster that divides the batch rows): every k block of a CTA in
  // flight at once; else a ring, two CTAs per SM
  if (tiles * p.ks <= a.sm_count && p.nb % p.ks == 0) return launch<kBlocks, kNBMax>(maps, p, tiles, s);
  return launch<3, kNBMax + kMaxCluster>(maps, p, tiles, s);
}

}  // namespace wv
