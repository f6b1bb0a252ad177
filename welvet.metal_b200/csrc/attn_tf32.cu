// Flash-attention prefill of the FP32 path on the tensor cores: 3xTF32 (x = hi +
// lo, hi the TF32 rounding of x, lo the FP32 remainder; a product is hi*hi + hi*lo
// + lo*hi, dropping lo*lo, 2^-22 relative), head_dim 64 — the FP32 replacement of
// the reference's single-thread attention loop (shaders/ops_mha.metal:31-127),
// within its 1e-4 budget.
//
// The QKV projection's epilogue writes the hi and lo parts of Q, K and V (RoPE
// applied). One CTA per (128-query tile, head, sequence), heaviest causal tiles
// first, 64 keys per block:
//   warps 0-7  two softmax warpgroups; warpgroup g owns the key blocks j == g
//              (mod 2) as an independent partial softmax (own running max, sum and
//              O accumulator), one query row per thread (its TMEM lane); the two
//              partial results are merged once, at the end
//   warp 8     TMA: Q (hi, lo) once, then K_j (hi, lo) into the K ring
//   warp 9     UMMA issuer (one thread): S_j = Qh Kh^T + Qh Kl^T + Ql Kh^T (SS,
//              kind::tf32) into TMEM buffer S_{j&1}; O_{j&1} += Ph V_h + Ph V_l +
//              Pl V_h as TS MMAs whose A operand is P in TMEM (Ph over S_j, Pl in
//              its own columns) and V an MN-major shared-memory operand (TMA
//              writes V in the 32-byte-atom 128-byte swizzle: MN-major TF32
//              operands take no other swizzled layout)
//   warp 10    TMA: V_j (hi, lo) into the V ring
// The softmax is the BF16 kernel's (attn_tc.cu): log2-domain online max and sum,
// masks evaluated only on blocks that straddle the mask edge (scores outside the
// row's allowed key interval set to -inf, then the unmasked code), lazy O rescale
// (threshold 2^8, exact since the final division uses the same reference maximum
// as every P); P is kept in FP32 and split into its TF32 hi and lo parts. The
// output row is written as FP32 and as the hi / lo split the O projection reads.
#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <climits>

namespace wv {
namespace {

constexpr int kHD = 64;     // head_dim
constexpr int kBQ = 128;    // query rows per tile
constexpr int kBK = 64;     // keys per block
constexpr int kSoftThreads = 256;
constexpr int kThreads = 384;  // warps 8-11: TMA Q/K (8), UMMA issuer (9), TMA V (10), idle (11)
constexpr int kLaunchRegs = 168;
constexpr int kLowRegs = 56;
constexpr int kHighRegs = 224;
static_assert(kLowRegs * 128 + kHighRegs * 256 <= kLaunchRegs * kThreads, "register split exceeds the pool");

// Shared memory: a 128-byte (32-float) wide column chunk of a tile, 128-byte
// swizzled as TMA writes it; head_dim 64 = two chunks. Each operand holds its hi
// chunks, then its lo chunks.
constexpr int kQChunk = kBQ * 128;  // 16 KB
constexpr int kKChunk = kBK * 128;  // 8 KB (K and V blocks alike)
constexpr int kQBytes = 4 * kQChunk;  // hi c0, hi c1, lo c0, lo c1
constexpr int kKBytes = 4 * kKChunk;
constexpr int kSK = 2, kSV = 2;  // ring depths
constexpr int kOffK = kQBytes;
constexpr int kOffV = kOffK + kSK * kKBytes;
constexpr int kOffEx = kOffK;  // final (max, sum) exchange, once the last S has run
constexpr int kOffBar = kOffV + kSV * kKBytes;
constexpr int kSmem = 1024 + kOffBar + 512;
static_assert(kSmem <= 227 * 1024, "shared memory");
// TMEM columns: S_g / Ph_g at 64 g, Pl_g at 128 + 64 g, O_g at 256 + 64 g.
constexpr uint32_t kColPl = 128, kColO = 256;

struct TParams {
  FParams f;
  float* out_hi;
  float* out_lo;
};

template <bool ALIBI, bool SIGMOID>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tf32_kernel(const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                     const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                     const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl,
                     const TParams tp) {
  const FParams& p = tp.f;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;
  uint64_t* k_empty = k_full + kSK;
  uint64_t* v_full = k_empty + kSK;
  uint64_t* v_empty = v_full + kSV;
  uint64_t* s_full = v_empty + kSV;  // [2] per warpgroup
  uint64_t* p_full = s_full + 2;     // [2] P written (and O rescaled)
  uint64_t* p_empty = p_full + 2;    // [2] PV complete
  uint64_t* fin_bar = p_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int qt = p.nqt - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int group = p.num_heads / p.num_kv_heads, kh = h / group;
  const int t0 = qt * kBQ;
  const int rows_here = min(kBQ, p.seq - t0);
  const int pos0 = p.stream_mode ? b * p.seq : 0;
  const int kv_end = p.stream_mode ? (b + 1) * p.seq : p.seq;
  const int q_row0 = b * p.seq + t0;
  const int key_row_base = p.stream_mode ? 0 : b * p.seq;
  int lo, hi;
  key_range(p, pos0 + t0, pos0 + t0 + rows_here - 1, kv_end, lo, hi);
  const int kb0 = (lo / kBK) * kBK;
  const int nblk = hi >= lo ? (hi - kb0) / kBK + 1 : 0;

  const int warp = (int)warp_id(), lane = (int)lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kSK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kSV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrival per warp of the warpgroup
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(fin_bar, kSoftThreads);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp >= 8) regs_dec<kLowRegs>();
  if (warp == 8) {
    // ------------------------------------------------------- producer: Q, K
    if (lane == 0 && nblk > 0) {
      tma_prefetch_desc(&tmQh);
      tma_prefetch_desc(&tmQl);
      tma_prefetch_desc(&tmKh);
      tma_prefetch_desc(&tmKl);
      mbar_arrive_expect_tx(q_full, kQBytes);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(smem + c * kQChunk, &tmQh, q_full, h * kHD + c * 32, q_row0);
        tma_load_2d(smem + (2 + c) * kQChunk, &tmQl, q_full, h * kHD + c * 32, q_row0);
      }
      for (int j = 0; j < nblk; ++j) {
        const int ks = j % kSK;
        if (!mbar_wait(&k_empty[ks], ((j / kSK) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&k_full[ks], kKBytes);
        const int krow = key_row_base + kb0 + j * kBK;
        uint8_t* dst = smem + kOffK + ks * kKBytes;
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(dst + c * kKChunk, &tmKh, &k_full[ks], kh * kHD + c * 32, krow);
          tma_load_2d(dst + (2 + c) * kKChunk, &tmKl, &k_full[ks], kh * kHD + c * 32, krow);
        }
      }
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------- producer: V
    if (lane == 0 && nblk > 0) {
      tma_prefetch_desc(&tmVh);
      tma_prefetch_desc(&tmVl);
      for (int i = 0; i < nblk; ++i) {
        const int vs = i % kSV;
        if (!mbar_wait(&v_empty[vs], ((i / kSV) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&v_full[vs], kKBytes);
        const int vrow = key_row_base + kb0 + i * kBK;
        uint8_t* dst = smem + kOffV + vs * kKBytes;
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(dst + c * kKChunk, &tmVh, &v_full[vs], kh * kHD + c * 32, vrow);
          tma_load_2d(dst + (2 + c) * kKChunk, &tmVl, &v_full[vs], kh * kHD + c * 32, vrow);
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- UMMA issuer
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t IDESC_S = idesc_make(2, kBQ, kBK, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_make(2, kBQ, kHD, 0, 1);
      constexpr uint32_t DHI = sdesc_hi_sw128(1024);
      constexpr uint32_t DHI_V = sdesc_hi_sw128_32b(4 * 128);
      if (!mbar_wait(q_full, 0, abort_flag, p.err, kErrWaitFull)) goto done;
      const uint32_t qh = sdesc_lo(smem_u32(smem), 16);
      const uint32_t ql = qh + (uint32_t)((2 * kQChunk) >> 4);
      // S_j: K-major A (Q) and B (K); a k-step is 8 TF32 values = 32 bytes of a
      // 128-byte row, four per chunk.
      auto issue_s = [&](int j) -> bool {
        const int ks = j % kSK, g = j & 1;
        if (!mbar_wait(&k_full[ks], (j / kSK) & 1, abort_flag, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t kh_ = sdesc_lo(smem_u32(smem + kOffK + ks * kKBytes), 16);
        const uint32_t kl_ = kh_ + (uint32_t)((2 * kKChunk) >> 4);
        const uint32_t d = tmem + (uint32_t)(g * kBK);
#pragma unroll
        for (int kk = 0; kk < kHD / 8; ++kk) {
          const uint32_t a_off = (uint32_t)(((kk >> 2) * kQChunk + (kk & 3) * 32) >> 4);
          const uint32_t b_off = (uint32_t)(((kk >> 2) * kKChunk + (kk & 3) * 32) >> 4);
          umma_tf32_ss_lohi(d, ql + a_off, kh_ + b_off, DHI, IDESC_S, kk > 0);
          umma_tf32_ss_lohi(d, qh + a_off, kl_ + b_off, DHI, IDESC_S, 1u);
          umma_tf32_ss_lohi(d, qh + a_off, kh_ + b_off, DHI, IDESC_S, 1u);
        }
        umma_commit(&k_empty[ks]);
        umma_commit(&s_full[g]);
        return true;
      };
      // PV_i: A = P from TMEM (a k-step is 8 keys = 8 columns), B = V MN-major in
      // the 32-byte-atom 128-byte swizzle: a k-step is 8 key rows of 128 bytes (two
      // 4-row swizzle groups, 512 bytes apart), the second 32-column chunk of
      // head_dim one chunk further (leading byte offset).
      auto issue_pv = [&](int i) -> bool {
        const int vs = i % kSV, g = i & 1;
        if (!mbar_wait(&p_full[g], (i >> 1) & 1, abort_flag, p.err, kErrWaitOther)) return false;
        if (!mbar_wait(&v_full[vs], (i / kSV) & 1, abort_flag, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t vh = sdesc_lo(smem_u32(smem + kOffV + vs * kKBytes), kKChunk);
        const uint32_t vl = vh + (uint32_t)((2 * kKChunk) >> 4);
        const uint32_t d = tmem + kColO + (uint32_t)(kHD * g);
        const uint32_t ph = tmem + (uint32_t)(g * kBK), pl = tmem + kColPl + (uint32_t)(g * kBK);
        const uint32_t acc0 = i >= 2 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          const uint32_t b_off = (uint32_t)((kk * 8 * 128) >> 4);
          umma_tf32_ts_lohi(d, pl + (uint32_t)(kk * 8), vh + b_off, DHI_V, IDESC_PV, kk > 0 ? 1u : acc0);
          umma_tf32_ts_lohi(d, ph + (uint32_t)(kk * 8), vl + b_off, DHI_V, IDESC_PV, 1u);
          umma_tf32_ts_lohi(d, ph + (uint32_t)(kk * 8), vh + b_off, DHI_V, IDESC_PV, 1u);
        }
        umma_commit(&v_empty[vs]);
        umma_commit(&p_empty[g]);
        return true;
      };
      for (int j = 0; j < min(2, nblk); ++j)
        if (!issue_s(j)) goto done;
      for (int i = 0; i < nblk; ++i) {
        if (!issue_pv(i)) goto done;
        if (i + 2 < nblk && !issue_s(i + 2)) goto done;
      }
    }
  } else if (warp < 8) {
    // -------------------------------------------------------------- softmax
    regs_inc<kHighRegs>();
    const int g = warp >> 2;
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;
    const int qpos = pos0 + t0 + r;
    const bool row_ok = r < rows_here;
    const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
    const uint32_t s_col = (uint32_t)(kBK * g), pl_col = kColPl + (uint32_t)(kBK * g),
                   o_col = kColO + (uint32_t)(kHD * g);
    const float sl = p.scale_log2;
    const float slope2 = ALIBI ? exp2f(-(float)(p.head_base + h + 1) * 8.0f / (float)p.total_heads) * kLog2e : 0.f;
    int row_lo = 0, row_hi = qpos;
    if (p.mask == 2) {
      row_hi = INT_MAX;
    } else if (p.mask == 3) {
      const int w = p.window > 0 ? p.window : p.msl;
      row_lo = qpos - w + 1;
      row_hi = p.window_causal ? qpos : qpos + w - 1;
    } else if (p.mask == 4 && qpos < p.prefix) {
      row_hi = max(qpos, p.prefix - 1);
    }
    row_hi = min(row_hi, kv_end - 1);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    int jl = -1;
    for (int j = g; j < nblk; j += 2) {
      ok = mbar_wait(&s_full[g], (j >> 1) & 1, abort_flag, p.err, kErrWaitAccFull);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[kBK];
#pragma unroll
      for (int c = 0; c < kBK / 32; ++c)
        tmem_ld32(tmem + lane_off + s_col + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&s[32 * c]));
      tmem_ld_wait();

      const int k0 = kb0 + j * kBK;
      const bool full = block_full(p, pos0 + t0, pos0 + t0 + kBQ - 1, k0, k0 + kBK - 1, kv_end);
      const bool fast = !ALIBI && sl > 0.f;
      if (fast && !full) {
        const int lo_rel = row_lo - k0, hi_rel = row_hi - k0;
#pragma unroll
        for (int i = 0; i < kBK; ++i)
          if (i < lo_rel || i > hi_rel) s[i] = 0xff800000u;  // -inf
      }
      float mx = -INFINITY;
      if (fast) {
        float m8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) m8[e] = fmaxf(__uint_as_float(s[e]), __uint_as_float(s[8 + e]));
#pragma unroll
        for (int i = 16; i < kBK; i += 16) {
#pragma unroll
          for (int e = 0; e < 8; ++e) m8[e] = fmax3(m8[e], __uint_as_float(s[i + e]), __uint_as_float(s[i + 8 + e]));
        }
        mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        mx *= sl;
      } else {
#pragma unroll
        for (int i = 0; i < kBK; ++i) {
          const int kpos = k0 + i;
          float v = __uint_as_float(s[i]) * sl;
          if (ALIBI) v -= slope2 * (float)abs(qpos - kpos);
          if (!full && !(kpos < kv_end && allow(p, qpos, kpos))) v = -INFINITY;
          s[i] = __float_as_uint(v);
          mx = fmaxf(mx, v);
        }
      }
      float corr = 1.f;
      bool need = false;
      if (!SIGMOID) {
        const float mnew = fmaxf(m, mx);
        if (m == -INFINITY) {
          m = mnew;
        } else if (mnew > m + kRescaleThreshold) {
          corr = fast_exp2(m - mnew);
          m = mnew;
          need = true;
        }
      }
      const float mref = (m == -INFINITY) ? 0.f : m;
      uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
      const uint64_t sl2 = f2pack(sl, sl), nm2 = f2pack(-mref, -mref);
      // P in FP32, stored as its TF32 hi part over S_g and its remainder in Pl_g,
      // 32 keys per store.
      auto exp_loop = [&](auto pair_fn) {
#pragma unroll
        for (int hh = 0; hh < kBK / 32; ++hh) {
          uint32_t ph[32], pl[32];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int i = 32 * hh + 2 * c;
            float a, c2;
            pair_fn(__uint_as_float(s[i]), __uint_as_float(s[i + 1]), a, c2);
            acc2[c & 3] = fadd2(acc2[c & 3], f2pack(a, c2));
            const float ah = to_tf32(a), ch = to_tf32(c2);
            ph[2 * c] = __float_as_uint(ah);
            ph[2 * c + 1] = __float_as_uint(ch);
            pl[2 * c] = __float_as_uint(a - ah);
            pl[2 * c + 1] = __float_as_uint(c2 - ch);
          }
          tmem_st32(tmem + lane_off + s_col + 32 * hh, ph);
          tmem_st32(tmem + lane_off + pl_col + 32 * hh, pl);
        }
      };
      if (SIGMOID) {
        const float k = fast ? sl : 1.f;
        exp_loop([&](float x0, float x1, float& a, float& c2) {
          const float v0 = x0 * k, v1 = x1 * k;
          a = v0 == -INFINITY ? 0.f : __frcp_rn(1.f + fast_exp2(-v0));
          c2 = v1 == -INFINITY ? 0.f : __frcp_rn(1.f + fast_exp2(-v1));
        });
      } else if (fast) {
        exp_loop([&](float x0, float x1, float& a, float& c2) {
          float y0, y1;
          f2unpack(ffma2(f2pack(x0, x1), sl2, nm2), y0, y1);
          a = fast_exp2(y0);
          c2 = fast_exp2(y1);
        });
      } else {
        exp_loop([&](float x0, float x1, float& a, float& c2) {
          float y0, y1;
          f2unpack(fadd2(f2pack(x0, x1), nm2), y0, y1);
          a = fast_exp2(y0);
          c2 = fast_exp2(y1);
        });
      }
      float r0, r1, r2, r3, r4, r5, r6, r7;
      f2unpack(acc2[0], r0, r1);
      f2unpack(acc2[1], r2, r3);
      f2unpack(acc2[2], r4, r5);
      f2unpack(acc2[3], r6, r7);
      l = l * corr + (((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)));
      if (!SIGMOID && __any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int c = 0; c < kHD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + o_col + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
          tmem_st32(tmem + lane_off + o_col + 32 * c, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
      jl = j;
    }
    // ---- merge the two partial softmaxes; warpgroup g writes output columns
    //      [32 g, 32 g + 32) of the row.
    if (ok && jl >= 0) ok = mbar_wait(&p_empty[g], (jl >> 1) & 1, abort_flag, p.err, kErrWaitOther);
    float* ex = reinterpret_cast<float*>(smem + kOffEx) + g * 256;
    const int nb_mine = g == 0 ? (nblk + 1) / 2 : nblk / 2, nb_other = g == 0 ? nblk / 2 : (nblk + 1) / 2;
    if (ok) {
      if (nb_mine > 0) {
        ex[r] = m;
        ex[128 + r] = l;
      }
      tc_fence_before();
      mbar_arrive(fin_bar);
      ok = mbar_wait(fin_bar, 0, abort_flag, p.err, kErrWaitOther);
    }
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const float* exo = reinterpret_cast<const float*>(smem + kOffEx) + (g ^ 1) * 256;
      const float mo = nb_other > 0 ? exo[r] : -INFINITY, lo_ = nb_other > 0 ? exo[128 + r] : 0.f;
      const float mA = g == 0 ? m : mo, lA = g == 0 ? l : lo_;
      const float mB = g == 0 ? mo : m, lB = g == 0 ? lo_ : l;
      const int nbA = (nblk + 1) / 2, nbB = nblk / 2;
      float wA = 1.f, wB = 1.f, inv = 1.f;
      if (!SIGMOID) {
        const float M = fmaxf(mA, mB);
        wA = (mA == -INFINITY) ? 0.f : fast_exp2(mA - M);
        wB = (mB == -INFINITY) ? 0.f : fast_exp2(mB - M);
        const float L = lA * wA + lB * wB;
        inv = L > 0.f ? 1.f / L : 0.f;
      }
      wA *= inv;
      wB *= inv;
      const uint32_t col = (uint32_t)(g * 32);
      uint32_t oa[32], ob[32];
      if (nbA > 0) tmem_ld32(tmem + lane_off + kColO + col, oa);
      if (nbB > 0) tmem_ld32(tmem + lane_off + kColO + kHD + col, ob);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int e = 0; e < 32; ++e)
        v[e] = (nbA > 0 ? __uint_as_float(oa[e]) * wA : 0.f) + (nbB > 0 ? __uint_as_float(ob[e]) * wB : 0.f);
      if (row_ok) {
        const size_t off = (size_t)(q_row0 + r) * p.ldo + (size_t)h * kHD + col;
        float* orow = static_cast<float*>(p.out) + off;
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          st_global_v4(orow + e, __float_as_uint(v[e]), __float_as_uint(v[e + 1]), __float_as_uint(v[e + 2]),
                       __float_as_uint(v[e + 3]));
        if (tp.out_hi) {
          float vh[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) vh[e] = to_tf32(v[e]);
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            st_global_v4(tp.out_hi + off + e, __float_as_uint(vh[e]), __float_as_uint(vh[e + 1]),
                         __float_as_uint(vh[e + 2]), __float_as_uint(vh[e + 3]));
            st_global_v4(tp.out_lo + off + e, __float_as_uint(v[e] - vh[e]), __float_as_uint(v[e + 1] - vh[e + 1]),
                         __float_as_uint(v[e + 2] - vh[e + 2]), __float_as_uint(v[e + 3] - vh[e + 3]));
          }
        }
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool ALIBI, bool SIGMOID>
cudaError_t launch_variant(const CUtensorMap* maps, const TParams& p, dim3 grid, cudaStream_t s) {
  auto kern = attn_tf32_kernel<ALIBI, SIGMOID>;
  static const cudaError_t ready = [kern]() {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa{};
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs * kThreads < kLowRegs * 128 + kHighRegs * 256) return cudaErrorNotSupported;
    return cudaSuccess;
  }();
  if (ready != cudaSuccess) return ready;
  kern<<<grid, kThreads, kSmem, s>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p);
  return cudaGetLastError();
}

} // namespace

bool attn_tf32_supported(const AttnArgs& a) {
  if (a.is_bf16 || a.head_dim != kHD || !a.q_lo || !a.k_lo || !a.v_lo) return false;
  if (a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads) return false;
  if (a.stream_mode && a.batch * a.seq > a.max_seq_len && a.batch > 1) return false;  // ring wrap
  if ((a.out_hi == nullptr) != (a.out_lo == nullptr)) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a.q) || !al16(a.k) || !al16(a.v) || !al16(a.q_lo) || !al16(a.k_lo) || !al16(a.v_lo)) return false;
  if (!al16(a.out) || (a.out_hi && (!al16(a.out_hi) || !al16(a.out_lo)))) return false;
  if ((a.ldq * 4) % 16 || (a.ldk * 4) % 16 || (a.ldo * 4) % 16) return false;
  return true;
}

cudaError_t attn_prefill_tf32(const AttnArgs& a, cudaStream_t s) {
  if (!attn_tf32_supported(a)) return cudaErrorInvalidValue;
  alignas(64) CUtensorMap maps[6];
  const int rows = a.batch * a.seq;
  const int qd = a.num_heads * kHD, kd = a.num_kv_heads * kHD;
  const int F32 = (int)CU_TENSOR_MAP_DATA_TYPE_FLOAT32, SW = (int)CU_TENSOR_MAP_SWIZZLE_128B;
  const int SWV = (int)CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;  // V is the MN-major operand
  if (!make_tma_2d(&maps[0], a.q, F32, 4, qd, rows, a.ldq, 32, kBQ, SW) ||
      !make_tma_2d(&maps[1], a.q_lo, F32, 4, qd, rows, a.ldq, 32, kBQ, SW) ||
      !make_tma_2d(&maps[2], a.k, F32, 4, kd, rows, a.ldk, 32, kBK, SW) ||
      !make_tma_2d(&maps[3], a.k_lo, F32, 4, kd, rows, a.ldk, 32, kBK, SW) ||
      !make_tma_2d(&maps[4], a.v, F32, 4, kd, rows, a.ldk, 32, kBK, SWV) ||
      !make_tma_2d(&maps[5], a.v_lo, F32, 4, kd, rows, a.ldk, 32, kBK, SWV))
    return cudaErrorInvalidValue;
  TParams p{};
  FParams& f = p.f;
  f.batch = a.batch;
  f.seq = a.seq;
  f.num_heads = a.num_heads;
  f.num_kv_heads = a.num_kv_heads;
  f.stream_mode = a.stream_mode;
  f.mask = a.mask;
  f.window = a.window;
  f.msl = a.max_seq_len;
  f.prefix = a.prefix_len;
  f.window_causal = a.window_causal;
  f.head_base = a.head_base;
  f.total_heads = a.total_heads > 0 ? a.total_heads : a.num_heads;
  f.scale_log2 = a.scale * kLog2e;
  f.out = a.out;
  f.ldo = a.ldo;
  f.nqt = (a.seq + kBQ - 1) / kBQ;
  f.err = a.err;
  p.out_hi = a.out_hi;
  p.out_lo = a.out_lo;
  dim3 grid(f.nqt, a.num_heads, a.batch);
  if (a.alibi)
    return a.sigmoid ? launch_variant<true, true>(maps, p, grid, s) : launch_variant<true, false>(maps, p, grid, s);
  return a.sigmoid ? launch_variant<false, true>(maps, p, grid, s) : launch_variant<false, false>(maps, p, grid, s);
}

} // namespace wv
