// Flash-attention prefill on the 5th-generation tensor cores (tcgen05), BF16
// inputs, FP32 accumulation, head_dim 64 or 128 — the B200 replacement for the
// reference's single-thread attention loop (shaders/ops_mha.metal:31-127).
//
// One CTA per (128-query tile, head, sequence), heaviest causal tiles first:
//   warps 0-7  two softmax warpgroups; warpgroup g owns the key blocks j == g
//              (mod 2) as an independent partial softmax (own running max, sum
//              and O accumulator) — one query row per thread, its TMEM lane. The
//              two partial results are merged once, at the end.
//   warp 8     TMA: Q once, then K_j (128 keys) into the K ring
//   warp 9     UMMA issuer (one thread): S_j = Q K_j^T (SS) into TMEM buffer
//              S_{j&1}; O_{j&1} += P_j V_j as a TS MMA whose A operand is P_j in
//              TMEM (V an MN-major shared-memory operand)
//   warp 10    TMA: V_j into the V ring
// Per block a warpgroup copies S_j into registers, scales, masks (attn_allow,
// ops_mha.metal:1-12, evaluated only on blocks that straddle the mask edge),
// applies ALiBi, keeps an online max/sum in the log2 domain and writes P_j as bf16
// pairs over the first 64 columns of S_j. Issue order S_0, S_1, then per block i:
// PV_i, S_{i+2}; MMAs of one thread run in order, so S_{i+2} overwrites the buffer
// only after PV_i has read P_i, and the arrival of S_{j+2} also tells the
// warpgroup that PV_j is done, i.e. O is current. O is rescaled only when a row
// maximum grows by more than 2^8 (exact: the final division uses the same
// reference maximum as every P). While one warpgroup works on block j the tensor
// core runs PV and S of the other's blocks.
#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <climits>

namespace wv {
namespace {

constexpr int kBQ = 128;  // query rows per tile
constexpr int kBK = 128;  // keys per block
constexpr int kSoftThreads = 256;  // warps 0-7: two softmax warpgroups
constexpr int kThreads = 384;      // warps 8-11: TMA Q/K (8), UMMA issuer (9), TMA V (10), idle (11)
// Register split by warpgroup (setmaxnreg): the launch gives every thread
// kLaunchRegs; the producer warpgroup drops to kLowRegs and the softmax
// warpgroups grow to kHighRegs. The host verifies the kernel's launch register
// count before the first launch so the split always fits the block's pool.
constexpr int kLaunchRegs = 168;
constexpr int kLowRegs = 56;
constexpr int kHighRegs = 224;
static_assert(kLowRegs * 128 + kHighRegs * 256 <= kLaunchRegs * kThreads, "register split exceeds the pool");
// Whether AttnArgs::pair = -1 (auto) picks the CTA-pair kernel where it applies.
constexpr bool kPairDefault = false;

// PAIR: a cluster of two CTAs (head_dim 128) shares each 128-key block: every
// UMMA is M = 256 (both CTAs' query tiles), issued by the leader CTA; CTA r holds
// keys [64 r, 64 r + 64) of the K block and head-dim columns [64 r, 64 r + 64) of
// the V block, so each SM stages and streams half of every K and V operand.
template <int HD, bool PAIR = false> struct FT {
  static_assert(!PAIR || HD == 128, "CTA pairs split head_dim into 128-byte halves");
  static constexpr int CH = HD / 64;            // 64-wide (128-byte) chunks of a row
  static constexpr int TILE = 128 * 128;        // bytes of a 128-row x 64-col bf16 chunk (16 KB)
  static constexpr int Q_BYTES = CH * TILE;
  static constexpr int K_ROWS = PAIR ? 64 : 128;   // keys of a K block held by this CTA
  static constexpr int K_CHUNK = K_ROWS * 128;     // bytes of one 64-column chunk of them
  static constexpr int K_BYTES = CH * K_CHUNK;
  static constexpr int V_BYTES = PAIR ? TILE : CH * TILE;  // 128 keys x (head_dim / 2 in a pair)
  static constexpr int SK = PAIR ? 4 : (HD == 128 ? 3 : 4);  // ring depths
  static constexpr int SV = PAIR ? 4 : (HD == 128 ? 3 : 4);
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + SK * K_BYTES;
  // Final (max, sum) exchange, 2 x 256 floats, in K stage 0: every S MMA (the last
  // reader of K) has completed before the last PV, which the exchange waits for.
  static constexpr int OFF_EX = OFF_K;
  static constexpr int OFF_BAR = OFF_V + SV * V_BYTES;
  static constexpr int SMEM = 1024 + OFF_BAR + 512;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(K_BYTES >= 2048, "exchange area");
};

template <int HD, bool ALIBI, bool SIGMOID, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FParams p) {
  using F = FT<HD, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + F::OFF_BAR);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;
  uint64_t* k_empty = k_full + F::SK;
  uint64_t* v_full = k_empty + F::SK;
  uint64_t* v_empty = v_full + F::SV;
  uint64_t* s_full = v_empty + F::SV;  // [2] per warpgroup
  uint64_t* p_full = s_full + 2;       // [2] P written over S (and O rescaled)
  uint64_t* p_empty = p_full + 2;      // [2] PV complete
  uint64_t* fin_bar = p_empty + 2;     // final (max, sum) exchange
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  // ---- work item: heaviest query tiles first
  const int qt = p.nqt - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int group = p.num_heads / p.num_kv_heads, kh = h / group;
  const int t0 = qt * kBQ;
  const int rows_here = min(kBQ, p.seq - t0);
  const int pos0 = p.stream_mode ? b * p.seq : 0;         // position of t = 0
  const int kv_end = p.stream_mode ? (b + 1) * p.seq : p.seq;
  const int q_row0 = b * p.seq + t0;                       // row in the Q matrix
  const int key_row_base = p.stream_mode ? 0 : b * p.seq;  // row of key position 0
  int lo, hi;
  // A pair runs the union of its two tiles' key ranges (tiles qt and qt - 1, leader
  // first); keys outside a CTA's own range are masked in its softmax.
  const bool leader = !PAIR || cluster_rank() == 0;
  const int rank_in_pair = PAIR && !leader ? 1 : 0;
  if (PAIR) {
    const int qt_lead = p.nqt - 1 - (int)(blockIdx.x & ~1u);
    key_range(p, pos0 + (qt_lead - 1) * kBQ, pos0 + min(p.seq, (qt_lead + 1) * kBQ) - 1, kv_end, lo, hi);
  } else {
    key_range(p, pos0 + t0, pos0 + t0 + rows_here - 1, kv_end, lo, hi);
  }
  const int kb0 = (lo / kBK) * kBK;
  const int nblk = hi >= lo ? (hi - kb0) / kBK + 1 : 0;

  const int warp = (int)warp_id(), lane = (int)lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < F::SK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < F::SV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      // one arrival per warp of the warpgroup (in a pair: of both CTAs' warpgroups,
      // on the leader's barrier)
      mbar_init(&p_full[i], PAIR ? 8 : 4);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(fin_bar, kSoftThreads);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    if (PAIR) {
      tmem_alloc_pair(tmem_holder, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  // In a pair the other CTA's loads and arrivals target this CTA's barriers: both
  // CTAs' barriers are initialised before either proceeds.
  if (PAIR) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // TMEM columns: S_g at 128*g (fp32, 128 keys); O_g at 256 + HD*g.

  if (warp >= 8) regs_dec<kLowRegs>();  // whole warpgroup 2, before any role branch
  if (warp == 8) {
    // ------------------------------------------------------- producer: Q, K
    if (lane == 0 && nblk > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      // In a pair the leader arms its barrier with both CTAs' bytes and both CTAs'
      // loads complete on it.
      if (leader) mbar_arrive_expect_tx(q_full, (PAIR ? 2 : 1) * F::Q_BYTES);
      for (int c = 0; c < F::CH; ++c) {
        if (PAIR) tma_load_2d_pair(smem + c * F::TILE, &tmQ, q_full, h * HD + c * 64, q_row0);
        else tma_load_2d(smem + c * F::TILE, &tmQ, q_full, h * HD + c * 64, q_row0);
      }
      for (int j = 0; j < nblk; ++j) {
        const int ks = j % F::SK;
        if (!mbar_wait(&k_empty[ks], ((j / F::SK) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        if (leader) mbar_arrive_expect_tx(&k_full[ks], (PAIR ? 2 : 1) * F::K_BYTES);
        const int krow = key_row_base + kb0 + j * kBK + rank_in_pair * F::K_ROWS;
        for (int c = 0; c < F::CH; ++c) {
          uint8_t* dst = smem + F::OFF_K + ks * F::K_BYTES + c * F::K_CHUNK;
          if (PAIR) tma_load_2d_pair(dst, &tmK, &k_full[ks], kh * HD + c * 64, krow);
          else tma_load_2d(dst, &tmK, &k_full[ks], kh * HD + c * 64, krow);
        }
      }
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------- producer: V
    // (its own thread: a V load never waits behind a K slot and vice versa)
    if (lane == 0 && nblk > 0) {
      tma_prefetch_desc(&tmV);
      for (int i = 0; i < nblk; ++i) {
        const int vs = i % F::SV;
        if (!mbar_wait(&v_empty[vs], ((i / F::SV) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        if (leader) mbar_arrive_expect_tx(&v_full[vs], (PAIR ? 2 : 1) * F::V_BYTES);
        uint8_t* dst = smem + F::OFF_V + vs * F::V_BYTES;
        if (PAIR) {  // head-dim columns [64 r, 64 r + 64) of the block
          tma_load_2d_pair(dst, &tmV, &v_full[vs], kh * HD + 64 * rank_in_pair, key_row_base + kb0 + i * kBK);
        } else {
          for (int c = 0; c < F::CH; ++c)
            tma_load_2d(dst + c * F::TILE, &tmV, &v_full[vs], kh * HD + c * 64, key_row_base + kb0 + i * kBK);
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- UMMA issuer
    if (lane == 0 && nblk > 0 && leader) {
      constexpr int MM = PAIR ? 2 * kBQ : kBQ;  // rows of one UMMA (both CTAs' tiles in a pair)
      constexpr uint32_t IDESC_S = idesc_make(1, MM, kBK, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_make(1, MM, HD, 0, 1);
      const uint32_t q_base = smem_u32(smem);
      if (!mbar_wait(q_full, 0, abort_flag, p.err, kErrWaitFull)) goto done;
      // S_j into TMEM buffer j&1 (columns 128*(j&1)); its warpgroup reads S_j into
      // registers and writes P_j (bf16 pairs) over the first 64 columns, which the
      // TS MMA of PV_j reads as its A operand. S_{j+2} reuses the buffer, so the
      // issue order is S_0, S_1, then per block i: PV_i, S_{i+2} (MMAs of one thread
      // execute in issue order).
      // Descriptors as 32-bit halves, advanced by constant adds (a short issue path
      // for the single issuing thread).
      constexpr uint32_t DHI = sdesc_hi_sw128(1024);
      const uint32_t q_lo = sdesc_lo(q_base, 16);
      auto issue_s = [&](int j) -> bool {
        const int ks = j % F::SK, g = j & 1;
        if (!mbar_wait(&k_full[ks], (j / F::SK) & 1, abort_flag, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t k_lo = sdesc_lo(smem_u32(smem + F::OFF_K + ks * F::K_BYTES), 16);
        const uint32_t d = tmem + (uint32_t)(g * 128);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t a_off = (uint32_t)(((kk >> 2) * F::TILE + (kk & 3) * 32) >> 4);
          const uint32_t b_off = (uint32_t)(((kk >> 2) * F::K_CHUNK + (kk & 3) * 32) >> 4);
          if (PAIR) umma2_f16_ss_lohi(d, q_lo + a_off, k_lo + b_off, DHI, IDESC_S, kk > 0);
          else umma_f16_ss_lohi(d, q_lo + a_off, k_lo + b_off, DHI, IDESC_S, kk > 0);
        }
        if (PAIR) {
          umma2_commit_both(&k_empty[ks]);
          umma2_commit_both(&s_full[g]);
        } else {
          umma_commit(&k_empty[ks]);
          umma_commit(&s_full[g]);
        }
        return true;
      };
      auto issue_pv = [&](int i) -> bool {
        const int vs = i % F::SV, g = i & 1;
        if (!mbar_wait(&p_full[g], (i >> 1) & 1, abort_flag, p.err, kErrWaitOther)) return false;
        if (!mbar_wait(&v_full[vs], (i / F::SV) & 1, abort_flag, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t v_lo = sdesc_lo(smem_u32(smem + F::OFF_V + vs * F::V_BYTES), F::TILE);
        const uint32_t d = tmem + (uint32_t)(256 + HD * g), pa = tmem + (uint32_t)(g * 128);
        const uint32_t acc0 = i >= 2 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // A = P from TMEM: 16 keys = 8 columns of bf16 pairs. V is MN-major: 16
          // keys = 16 rows of 128 bytes; the second 64-column chunk of head_dim
          // sits one TILE further (leading byte offset; in a pair each CTA holds
          // one 64-column chunk, the other CTA's half of N).
          const uint32_t b = v_lo + (uint32_t)((kk * 16 * 128) >> 4);
          if (PAIR) umma2_f16_ts_lohi(d, pa + (uint32_t)(kk * 8), b, DHI, IDESC_PV, kk > 0 ? 1u : acc0);
          else umma_f16_ts_lohi(d, pa + (uint32_t)(kk * 8), b, DHI, IDESC_PV, kk > 0 ? 1u : acc0);
        }
        if (PAIR) {
          umma2_commit_both(&v_empty[vs]);
          umma2_commit_both(&p_empty[g]);
        } else {
          umma_commit(&v_empty[vs]);
          umma_commit(&p_empty[g]);
        }
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
    const int g = warp >> 2;  // this warpgroup owns blocks j == g (mod 2)
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;   // query row within the tile (= TMEM lane)
    const int qpos = pos0 + t0 + r;
    const bool row_ok = r < rows_here;
    const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
    const uint32_t s_col = (uint32_t)(128 * g), o_col = (uint32_t)(256 + HD * g);
    const float sl = p.scale_log2;
    const float slope2 = ALIBI ? exp2f(-(float)(p.head_base + h + 1) * 8.0f / (float)p.total_heads) * kLog2e : 0.f;
    // The keys attn_allow admits for this row form one interval [row_lo, row_hi]
    // (causal: [0, q]; sliding window: [q-w+1, q] or (q-w, q+w); prefix-LM:
    // [0, max(q, prefix-1)] inside the prefix), cut at the end of the keys.
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
    int jl = -1;  // last block processed by this warpgroup
    for (int j = g; j < nblk; j += 2) {
      ok = mbar_wait(&s_full[g], (j >> 1) & 1, abort_flag, p.err, kErrWaitAccFull);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld32(tmem + lane_off + s_col + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&s[32 * c]));
      tmem_ld_wait();

      const int k0 = kb0 + j * kBK;
      const bool full = block_full(p, pos0 + t0, pos0 + t0 + kBQ - 1, k0, k0 + kBK - 1, kv_end);
      // Fast path (no ALiBi, positive scale): logits are s * sl and the max of the
      // logits is sl * max(s). A block that straddles the mask edge first sets the
      // raw scores outside the row's interval to -inf (one compare and select per
      // score; -inf * sl stays -inf) and then takes the same code as an unmasked
      // block: a separate masked variant of the loops ran once per tile and paid
      // for its instruction fetches every time (about 25k cycles against 2.3k).
      const bool fast = !ALIBI && sl > 0.f;
      if (fast && !full) {
        const int lo_rel = row_lo - k0, hi_rel = row_hi - k0;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i < lo_rel || i > hi_rel) s[i] = 0xff800000u;  // -inf
      }
      float mx = -INFINITY;
      if (fast) {
        float m8[8];  // independent partial maxima (ILP), three-input max
#pragma unroll
        for (int e = 0; e < 8; ++e) m8[e] = fmaxf(__uint_as_float(s[e]), __uint_as_float(s[8 + e]));
#pragma unroll
        for (int i = 16; i < 128; i += 16) {
#pragma unroll
          for (int e = 0; e < 8; ++e) m8[e] = fmax3(m8[e], __uint_as_float(s[i + e]), __uint_as_float(s[i + 8 + e]));
        }
        mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        mx *= sl;
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
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
          m = mnew;  // first allowed keys of the row: nothing accumulated yet
        } else if (mnew > m + kRescaleThreshold) {
          corr = fast_exp2(m - mnew);
          m = mnew;
          need = true;
        }
      }
      const float mref = (m == -INFINITY) ? 0.f : m;
      // O_g is current: S_j completed after PV_{j-2} (issue order), and s_full(j)
      // covers every MMA issued before it.
      uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};  // packed partial row sums (ILP)
      const uint64_t sl2 = f2pack(sl, sl), nm2 = f2pack(-mref, -mref);
      // One loop per case (the case is uniform over the block): a per-pair branch
      // inside the unrolled loop would cost a branch and its resolution per pair.
      // P as bf16 pairs over columns [0, 64) of S_g, 32 columns (64 keys) per store.
      auto exp_loop = [&](auto pair_fn) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t pk[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int i = 64 * hh + 2 * c;
            float a, c2;
            pair_fn(__uint_as_float(s[i]), __uint_as_float(s[i + 1]), a, c2);
            acc2[c & 3] = fadd2(acc2[c & 3], f2pack(a, c2));
            pk[c] = pack_bf16x2(a, c2);
          }
          tmem_st32(tmem + lane_off + s_col + 32 * hh, pk);
        }
      };
      if (SIGMOID) {
        const float k = fast ? sl : 1.f;  // masked logits are already scaled
        exp_loop([&](float x0, float x1, float& a, float& c2) {
          const float v0 = x0 * k, v1 = x1 * k;
          a = v0 == -INFINITY ? 0.f : __frcp_rn(1.f + fast_exp2(-v0));
          c2 = v1 == -INFINITY ? 0.f : __frcp_rn(1.f + fast_exp2(-v1));
        });
      } else if (fast) {
        exp_loop([&](float x0, float x1, float& a, float& c2) {
          float y0, y1;  // logits x*sl - m as one packed FMA
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
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + o_col + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
          tmem_st32(tmem + lane_off + o_col + 32 * c, o);
        }
      }
      // Each thread's TMEM stores complete before its fence; the warp converges and
      // one lane arrives (four arrivals per warpgroup instead of 128 on the MMA
      // issuer's critical path).
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        // the leader's issuer waits for P in both CTAs' TMEM
        if (PAIR) mbar_arrive_leader(&p_full[g]);
        else mbar_arrive(&p_full[g]);
      }
      jl = j;
    }
    // ---- merge the two partial softmaxes; warpgroup g writes output columns
    //      [g*HD/2, (g+1)*HD/2) of the row.
    if (ok && jl >= 0) ok = mbar_wait(&p_empty[g], (jl >> 1) & 1, abort_flag, p.err, kErrWaitOther);
    float* ex = reinterpret_cast<float*>(smem + F::OFF_EX) + g * 256;
    // A warpgroup without blocks (warpgroup 1 when nblk <= 1) writes nothing: the
    // exchange lies in the K ring, which is only free once the last S has run.
    const int nb_mine = g == 0 ? (nblk + 1) / 2 : nblk / 2, nb_other = g == 0 ? nblk / 2 : (nblk + 1) / 2;
    if (ok) {
      if (nb_mine > 0) {
        ex[r] = m;
        ex[128 + r] = l;
      }
      // The other warpgroup reads O_g after this arrive; it orders after the
      // p_empty[g] completion observed above (release/acquire through fin_bar).
      tc_fence_before();
      mbar_arrive(fin_bar);
      ok = mbar_wait(fin_bar, 0, abort_flag, p.err, kErrWaitOther);
    }
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const float* exo = reinterpret_cast<const float*>(smem + F::OFF_EX) + (g ^ 1) * 256;
      const float mo = nb_other > 0 ? exo[r] : -INFINITY, lo = nb_other > 0 ? exo[128 + r] : 0.f;
      const float mA = g == 0 ? m : mo, lA = g == 0 ? l : lo;
      const float mB = g == 0 ? mo : m, lB = g == 0 ? lo : l;
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
      __nv_bfloat16* orow =
          static_cast<__nv_bfloat16*>(p.out) + (size_t)(q_row0 + r) * p.ldo + (size_t)h * HD + g * (HD / 2);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        const uint32_t col = (uint32_t)(g * (HD / 2) + 32 * c);
        uint32_t oa[32], ob[32];
        if (nbA > 0) tmem_ld32(tmem + lane_off + 256 + col, oa);
        if (nbB > 0) tmem_ld32(tmem + lane_off + 256 + HD + col, ob);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e)
          v[e] = (nbA > 0 ? __uint_as_float(oa[e]) * wA : 0.f) + (nbB > 0 ? __uint_as_float(ob[e]) * wB : 0.f);
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 8)
            st_global_v4(orow + 32 * c + e, pack_bf16x2(v[e], v[e + 1]), pack_bf16x2(v[e + 2], v[e + 3]),
                         pack_bf16x2(v[e + 4], v[e + 5]), pack_bf16x2(v[e + 6], v[e + 7]));
        }
      }
    }
  }
done:
  tc_fence_before();
  // In a pair neither CTA leaves (and frees shared memory or TMEM the leader's
  // MMAs or the other CTA's loads and arrivals use) before both are done.
  if (PAIR) cluster_sync();
  else __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem, 512);
    else tmem_dealloc(tmem, 512);
  }
}

template <int HD, bool ALIBI, bool SIGMOID, bool PAIR>
cudaError_t launch_variant(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FParams& p,
                           dim3 grid, cudaStream_t s) {
  using F = FT<HD, PAIR>;
  auto kern = attn_fwd_kernel<HD, ALIBI, SIGMOID, PAIR>;
  static const cudaError_t ready = [kern]() {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, F::SMEM);
    if (e != cudaSuccess) return e;
    // setmaxnreg.inc waits until the block's register pool can serve it: refuse to
    // launch unless the pool (launch registers x threads) covers the split.
    cudaFuncAttributes fa{};
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs * kThreads < kLowRegs * 128 + kHighRegs * 256) return cudaErrorNotSupported;
    return cudaSuccess;
  }();
  if (ready != cudaSuccess) return ready;
  if (!PAIR) {
    kern<<<grid, kThreads, F::SMEM, s>>>(mq, mk, mv, p);
    return cudaGetLastError();
  }
  // CTA pairs: clusters of two consecutive query tiles of one (head, sequence)
  cudaLaunchConfig_t lc{};
  lc.gridDim = grid;
  lc.blockDim = dim3(kThreads, 1, 1);
  lc.dynamicSmemBytes = F::SMEM;
  lc.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, kern, mq, mk, mv, p);
}

template <int HD, bool PAIR> cudaError_t launch(const AttnArgs& a, cudaStream_t s) {
  alignas(64) CUtensorMap mq, mk, mv;
  const int rows = a.batch * a.seq;
  const int qd = a.num_heads * HD, kd = a.num_kv_heads * HD;
  const int BF16 = (int)CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, SW = (int)CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_tma_2d(&mq, a.q, BF16, 2, qd, rows, a.ldq, 64, 128, SW) ||
      !make_tma_2d(&mk, a.k, BF16, 2, kd, rows, a.ldk, 64, FT<HD, PAIR>::K_ROWS, SW) ||
      !make_tma_2d(&mv, a.v, BF16, 2, kd, rows, a.ldk, 64, 128, SW))
    return cudaErrorInvalidValue;
  FParams p{};
  p.batch = a.batch;
  p.seq = a.seq;
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.stream_mode = a.stream_mode;
  p.mask = a.mask;
  p.window = a.window;
  p.msl = a.max_seq_len;
  p.prefix = a.prefix_len;
  p.window_causal = a.window_causal;
  p.head_base = a.head_base;
  p.total_heads = a.total_heads > 0 ? a.total_heads : a.num_heads;
  p.scale_log2 = a.scale * kLog2e;
  p.out = a.out;
  p.ldo = a.ldo;
  p.nqt = (a.seq + kBQ - 1) / kBQ;
  p.err = a.err;
  dim3 grid(p.nqt, a.num_heads, a.batch);
  if (a.alibi)
    return a.sigmoid ? launch_variant<HD, true, true, PAIR>(mq, mk, mv, p, grid, s)
                     : launch_variant<HD, true, false, PAIR>(mq, mk, mv, p, grid, s);
  return a.sigmoid ? launch_variant<HD, false, true, PAIR>(mq, mk, mv, p, grid, s)
                   : launch_variant<HD, false, false, PAIR>(mq, mk, mv, p, grid, s);
}

} // namespace

bool attn_tc_supported(const AttnArgs& a) {
  if (!a.is_bf16 || (a.head_dim != 64 && a.head_dim != 128)) return false;
  if (a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads) return false;
  // The ring-wrapped stream case (keys gathered from ring slots) stays on the
  // CUDA-core kernel; so do outputs that need a TF32 split.
  if (a.stream_mode && a.batch * a.seq > a.max_seq_len && a.batch > 1) return false;
  if (a.out_hi) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a.q) || !al16(a.k) || !al16(a.v) || !al16(a.out)) return false;
  if ((a.ldq * 2) % 16 || (a.ldk * 2) % 16 || (a.ldo * 2) % 16) return false;
  return true;
}

bool attn_tc_pair_supported(const AttnArgs& a) {
  // head_dim 128 (each CTA holds a 128-byte half of V's rows) and whole pairs of
  // 128-query tiles per sequence
  return attn_tc_supported(a) && a.head_dim == 128 && a.seq % (2 * kBQ) == 0;
}

cudaError_t attn_prefill_tc(const AttnArgs& a, cudaStream_t s) {
  if (!attn_tc_supported(a)) return cudaErrorInvalidValue;
  const bool pair = a.pair > 0 || (a.pair < 0 && kPairDefault && attn_tc_pair_supported(a));
  if (!pair && a.tile_ctr) return attn_prefill_persist(a, s);
  if (pair) {
    if (!attn_tc_pair_supported(a)) return cudaErrorInvalidValue;
    return launch<128, true>(a, s);
  }
  return a.head_dim == 64 ? launch<64, false>(a, s) : launch<128, false>(a, s);
}

} // namespace wv
