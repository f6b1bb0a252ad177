// Persistent flash-attention prefill on the tensor cores (tcgen05), BF16 inputs,
// FP32 accumulation, head_dim 64 or 128: the default form of the BF16 prefill
// attention (the reference's single-thread loop, shaders/ops_mha.metal:31-127).
//
// The per-tile pipeline is the one of attn_tc.cu's kernel (two softmax warpgroups
// on alternate 128-key blocks, S = Q K^T by SS UMMA into two TMEM buffers, P as
// bf16 over S, O += P V by TS UMMA, lazy O rescale, partial softmaxes merged at the
// end). What changes is the life of a CTA: one CTA per SM loops over (128-query
// tile, head, sequence) work items taken from a global counter, so the end of one
// tile overlaps the start of the next instead of leaving the tensor core idle:
//   * a scheduler thread (warp 11) fetches tile indices one ahead into a
//     two-slot queue in shared memory;
//   * the TMA producers run ahead into the next tile: its Q is loaded as soon as
//     the last S MMA of the current tile has read the Q buffer (q_empty), its
//     first K/V blocks as soon as ring slots free up;
//   * the MMA thread issues the next tile's first two S MMAs right behind the
//     current tile's last PV; only the next tile's first PV (which overwrites the
//     O accumulators) waits until the softmax warps have read O (o_free);
//   * the output rows are normalised in registers, written to shared memory and
//     stored by one TMA store per warpgroup (the softmax warps do not wait for it).
// Work items are ordered (sequence, head)-major with the heaviest causal query
// tiles of each head first, so the tiles resident at one time share a few heads'
// K/V in L2 and the light tiles end the launch. Block parities (S buffer, K/V
// ring slot, barrier phase) run on per-CTA counters across tiles.
#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <climits>

namespace wv {
namespace {

constexpr int kBQ = 128;  // query rows per tile
constexpr int kBK = 128;  // keys per block
constexpr int kSoftThreads = 256;
constexpr int kThreads = 384;  // warps 8-11: TMA Q/K (8), UMMA (9), TMA V (10), tile scheduler (11)
constexpr int kLaunchRegs = 168;
constexpr int kLowRegs = 56;
constexpr int kHighRegs = 224;
static_assert(kLowRegs * 128 + kHighRegs * 256 <= kLaunchRegs * kThreads, "register split exceeds the pool");
// Arrivals that release a tile-queue slot: Q/K producer, V producer, MMA thread and
// one per softmax warp.
constexpr int kTileConsumers = 3 + kSoftThreads / 32;

template <int HD> struct PT {
  static constexpr int CH = HD / 64;          // 128-byte (64-column) chunks of a row
  static constexpr int TILE = 128 * 128;      // one 128-row x 128-byte chunk
  static constexpr int Q_BYTES = CH * TILE;
  static constexpr int K_BYTES = CH * TILE;   // 128 keys
  static constexpr int V_BYTES = CH * TILE;
  static constexpr int SK = HD == 128 ? 2 : 4;  // ring depths
  static constexpr int SV = SK;
  static constexpr int OUT_HALF = 128 * HD;   // a warpgroup's output: 128 rows x HD/2 bf16
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + SK * K_BYTES;
  static constexpr int OFF_OUT = OFF_V + SV * V_BYTES;
  static constexpr int OFF_EX = OFF_OUT + 2 * OUT_HALF;  // (max, sum) exchange, 2 x 256 floats
  static constexpr int OFF_BAR = OFF_EX + 2048;
  static constexpr int SMEM = 1024 + OFF_BAR + 512;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// One work item: tile index -> (sequence, head, query tile) and the key blocks the
// tile's rows may see.
struct Tile {
  int b, h, kh, t0, rows_here, pos0, kv_end, q_row0, key_row_base, kb0, nblk;
};
__device__ __forceinline__ Tile tile_of(const FParams& p, int t) {
  Tile w;
  const int bh = t / p.nqt;
  const int qt = p.nqt - 1 - t % p.nqt;  // heaviest causal tile of the head first
  w.h = bh % p.num_heads;
  w.b = bh / p.num_heads;
  w.kh = w.h / (p.num_heads / p.num_kv_heads);
  w.t0 = qt * kBQ;
  w.rows_here = min(kBQ, p.seq - w.t0);
  w.pos0 = p.stream_mode ? w.b * p.seq : 0;
  w.kv_end = p.stream_mode ? (w.b + 1) * p.seq : p.seq;
  w.q_row0 = w.b * p.seq + w.t0;
  w.key_row_base = p.stream_mode ? 0 : w.b * p.seq;
  int lo, hi;
  key_range(p, w.pos0 + w.t0, w.pos0 + w.t0 + w.rows_here - 1, w.kv_end, lo, hi);
  w.kb0 = (lo / kBK) * kBK;
  w.nblk = hi >= lo ? (hi - w.kb0) / kBK + 1 : 0;
  return w;
}

template <int HD, bool ALIBI, bool SIGMOID>
__global__ void __launch_bounds__(kThreads, 1)
    attn_persist_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                        const FParams p, int* tile_ctr, int ntiles) {
  using F = PT<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + F::OFF_BAR);
  uint64_t* q_full = bar;
  uint64_t* q_empty = bar + 1;       // the tile's last S MMA has read Q
  uint64_t* k_full = bar + 2;
  uint64_t* k_empty = k_full + F::SK;
  uint64_t* v_full = k_empty + F::SK;
  uint64_t* v_empty = v_full + F::SV;
  uint64_t* s_full = v_empty + F::SV;  // [2] per warpgroup
  uint64_t* p_full = s_full + 2;       // [2] P written over S (and O rescaled)
  uint64_t* p_empty = p_full + 2;      // [2] PV complete
  uint64_t* fin_bar = p_empty + 2;     // (max, sum) exchange of a tile
  uint64_t* o_free = fin_bar + 1;      // the softmax warps have read the tile's O
  uint64_t* tile_full = o_free + 1;    // [2] tile queue
  uint64_t* tile_empty = tile_full + 2;
  uint64_t* stage_bar = tile_empty + 2;  // [2] a warpgroup's output rows staged
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stage_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* tile_slot = reinterpret_cast<volatile int*>(tmem_holder + 2);  // [2]

  const int warp = (int)warp_id(), lane = (int)lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
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
      mbar_init(&p_full[i], 4);  // one arrival per warp of the warpgroup
      mbar_init(&p_empty[i], 1);
      mbar_init(&tile_full[i], 1);
      mbar_init(&tile_empty[i], kTileConsumers);
      mbar_init(&stage_bar[i], 4);  // one arrival per warp of the warpgroup
    }
    mbar_init(fin_bar, kSoftThreads);
    mbar_init(o_free, kSoftThreads / 32);
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
  // TMEM columns: S_g at 128 g (fp32, 128 keys; P as bf16 pairs over its first 64);
  // O_g at 256 + HD g.

  // k-th entry of the tile queue (every role reads every entry in order).
  auto fetch = [&](int k, int& t) -> bool {
    if (!mbar_wait(&tile_full[k & 1], (k >> 1) & 1, abort_flag, p.err, kErrWaitOther)) return false;
    t = tile_slot[k & 1];
    return true;
  };

  if (warp >= 8) regs_dec<kLowRegs>();
  if (warp == 11) {
    // ------------------------------------------------------- tile scheduler
    if (lane == 0) {
      for (int k = 0;; ++k) {
        const int s = k & 1;
        if (k >= 2 && !mbar_wait(&tile_empty[s], ((k >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        const int t = atomicAdd(tile_ctr, 1);
        tile_slot[s] = t;
        mbar_arrive(&tile_full[s]);  // release: the slot is visible to the waiters
        if (t >= ntiles) break;
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------- producer: Q, K
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      int kb = 0, qi = 0;
      for (int k = 0;; ++k) {
        int t;
        if (!fetch(k, t)) break;
        mbar_arrive(&tile_empty[k & 1]);
        if (t >= ntiles) break;
        const Tile w = tile_of(p, t);
        if (w.nblk == 0) continue;
        if (qi > 0 && !mbar_wait(q_empty, (qi - 1) & 1, abort_flag, p.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(q_full, F::Q_BYTES);
        for (int c = 0; c < F::CH; ++c) tma_load_2d(smem + c * F::TILE, &tmQ, q_full, w.h * HD + c * 64, w.q_row0);
        ++qi;
        bool ok = true;
        for (int j = 0; j < w.nblk; ++j, ++kb) {
          const int ks = kb % F::SK;
          if (!mbar_wait(&k_empty[ks], ((kb / F::SK) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[ks], F::K_BYTES);
          const int krow = w.key_row_base + w.kb0 + j * kBK;
          for (int c = 0; c < F::CH; ++c)
            tma_load_2d(smem + F::OFF_K + ks * F::K_BYTES + c * F::TILE, &tmK, &k_full[ks], w.kh * HD + c * 64, krow);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------- producer: V
    if (lane == 0) {
      tma_prefetch_desc(&tmV);
      int vb = 0;
      for (int k = 0;; ++k) {
        int t;
        if (!fetch(k, t)) break;
        mbar_arrive(&tile_empty[k & 1]);
        if (t >= ntiles) break;
        const Tile w = tile_of(p, t);
        bool ok = true;
        for (int i = 0; i < w.nblk; ++i, ++vb) {
          const int vs = vb % F::SV;
          if (!mbar_wait(&v_empty[vs], ((vb / F::SV) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[vs], F::V_BYTES);
          const int vrow = w.key_row_base + w.kb0 + i * kBK;
          for (int c = 0; c < F::CH; ++c)
            tma_load_2d(smem + F::OFF_V + vs * F::V_BYTES + c * F::TILE, &tmV, &v_full[vs], w.kh * HD + c * 64, vrow);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- UMMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_make(1, kBQ, kBK, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_make(1, kBQ, HD, 0, 1);
      constexpr uint32_t DHI = sdesc_hi_sw128(1024);
      const uint32_t q_lo = sdesc_lo(smem_u32(smem), 16);
      int kb = 0, vb = 0, gb = 0, qi = 0;
      for (int k = 0;; ++k) {
        int t;
        if (!fetch(k, t)) break;
        mbar_arrive(&tile_empty[k & 1]);
        if (t >= ntiles) break;
        const int nblk = tile_of(p, t).nblk;
        if (nblk == 0) continue;
        if (!mbar_wait(q_full, qi & 1, abort_flag, p.err, kErrWaitFull)) break;
        ++qi;
        // S_j of block j (global block gb + j) into TMEM buffer (gb + j) & 1; the
        // tile's last S also releases Q to the producer.
        auto issue_s = [&](int j) -> bool {
          const int kbj = kb + j, ks = kbj % F::SK, g = (gb + j) & 1;
          if (!mbar_wait(&k_full[ks], (kbj / F::SK) & 1, abort_flag, p.err, kErrWaitFull)) return false;
          tc_fence_after();
          const uint32_t k_lo = sdesc_lo(smem_u32(smem + F::OFF_K + ks * F::K_BYTES), 16);
          const uint32_t d = tmem + (uint32_t)(g * 128);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (uint32_t)(((kk >> 2) * F::TILE + (kk & 3) * 32) >> 4);
            umma_f16_ss_lohi(d, q_lo + off, k_lo + off, DHI, IDESC_S, kk > 0);
          }
          umma_commit(&k_empty[ks]);
          umma_commit(&s_full[g]);
          if (j == nblk - 1) umma_commit(q_empty);
          return true;
        };
        // PV_i accumulates into O_g; the first PV of each buffer in the tile
        // overwrites it, so the tile's first PV waits until the previous tile's
        // epilogue has read both O buffers.
        auto issue_pv = [&](int i) -> bool {
          const int gbi = gb + i, g = gbi & 1, vbi = vb + i, vs = vbi % F::SV;
          if (i == 0 && k > 0 && !mbar_wait(o_free, (k - 1) & 1, abort_flag, p.err, kErrWaitOther)) return false;
          if (!mbar_wait(&p_full[g], (gbi >> 1) & 1, abort_flag, p.err, kErrWaitOther)) return false;
          if (!mbar_wait(&v_full[vs], (vbi / F::SV) & 1, abort_flag, p.err, kErrWaitFull)) return false;
          tc_fence_after();
          const uint32_t v_lo = sdesc_lo(smem_u32(smem + F::OFF_V + vs * F::V_BYTES), F::TILE);
          const uint32_t d = tmem + (uint32_t)(256 + HD * g), pa = tmem + (uint32_t)(g * 128);
          const uint32_t acc0 = i >= 2 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t b = v_lo + (uint32_t)((kk * 16 * 128) >> 4);
            umma_f16_ts_lohi(d, pa + (uint32_t)(kk * 8), b, DHI, IDESC_PV, kk > 0 ? 1u : acc0);
          }
          umma_commit(&v_empty[vs]);
          umma_commit(&p_empty[g]);
          return true;
        };
        bool ok = true;
        for (int j = 0; ok && j < min(2, nblk); ++j) ok = issue_s(j);
        for (int i = 0; ok && i < nblk; ++i) {
          ok = issue_pv(i);
          if (ok && i + 2 < nblk) ok = issue_s(i + 2);
        }
        if (!ok) break;
        kb += nblk;
        vb += nblk;
        gb += nblk;
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    regs_inc<kHighRegs>();
    const int g = warp >> 2;   // this warpgroup owns the global blocks of parity g
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;  // query row within the tile (= TMEM lane)
    const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
    const uint32_t s_col = (uint32_t)(128 * g), o_col = (uint32_t)(256 + HD * g);
    const float sl = p.scale_log2;
    const bool fast = !ALIBI && sl > 0.f;
    int gb = 0;        // global blocks of the tiles before this one
    int n_staged = 0;  // tiles whose rows this warpgroup staged for a TMA store
    for (int k = 0;; ++k) {
      int t;
      const bool got = fetch(k, t);
      if (!__all_sync(0xffffffffu, got)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&tile_empty[k & 1]);
      if (t >= ntiles) break;
      const Tile w = tile_of(p, t);
      const int qpos = w.pos0 + w.t0 + r;
      const float slope2 =
          ALIBI ? exp2f(-(float)(p.head_base + w.h + 1) * 8.0f / (float)p.total_heads) * kLog2e : 0.f;
      // The keys attn_allow admits for this row form one interval [row_lo, row_hi],
      // cut at the end of the keys.
      int row_lo = 0, row_hi = qpos;
      if (p.mask == 2) {
        row_hi = INT_MAX;
      } else if (p.mask == 3) {
        const int wdw = p.window > 0 ? p.window : p.msl;
        row_lo = qpos - wdw + 1;
        row_hi = p.window_causal ? qpos : qpos + wdw - 1;
      } else if (p.mask == 4 && qpos < p.prefix) {
        row_hi = max(qpos, p.prefix - 1);
      }
      row_hi = min(row_hi, w.kv_end - 1);
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      int jl = -1, nb_mine = 0;
      for (int j = ((gb & 1) == g) ? 0 : 1; j < w.nblk; j += 2) {
        const int gbj = gb + j;
        ok = mbar_wait(&s_full[g], (gbj >> 1) & 1, abort_flag, p.err, kErrWaitAccFull);
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

        const int k0 = w.kb0 + j * kBK;
        const bool full = block_full(p, w.pos0 + w.t0, w.pos0 + w.t0 + kBQ - 1, k0, k0 + kBK - 1, w.kv_end);
        // Fast path (no ALiBi, positive scale): a block that straddles the mask edge
        // first sets the raw scores outside the row's interval to -inf, then takes
        // the unmasked code.
        if (fast && !full) {
          const int lo_rel = row_lo - k0, hi_rel = row_hi - k0;
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i < lo_rel || i > hi_rel) s[i] = 0xff800000u;  // -inf
        }
        float mx = -INFINITY;
        if (fast) {
          float m8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) m8[e] = fmaxf(__uint_as_float(s[e]), __uint_as_float(s[8 + e]));
#pragma unroll
          for (int i = 16; i < 128; i += 16) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              m8[e] = fmax3(m8[e], __uint_as_float(s[i + e]), __uint_as_float(s[i + 8 + e]));
          }
          mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
          mx *= sl;
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            const int kpos = k0 + i;
            float v = __uint_as_float(s[i]) * sl;
            if (ALIBI) v -= slope2 * (float)abs(qpos - kpos);
            if (!full && !(kpos < w.kv_end && allow(p, qpos, kpos))) v = -INFINITY;
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
          const float kk = fast ? sl : 1.f;  // masked logits are already scaled
          exp_loop([&](float x0, float x1, float& a, float& c2) {
            const float v0 = x0 * kk, v1 = x1 * kk;
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
          for (int c = 0; c < HD / 32; ++c) {
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
        jl = gbj;
        ++nb_mine;
      }
      // ---- merge the two partial softmaxes; warpgroup g writes output columns
      //      [g HD/2, (g+1) HD/2) of the tile's rows.
      if (ok && jl >= 0) ok = mbar_wait(&p_empty[g], (jl >> 1) & 1, abort_flag, p.err, kErrWaitOther);
      // (tile values recomputed rather than kept live through the block loop)
      const Tile we = tile_of(p, t);
      const bool store_thread = threadIdx.x == (unsigned)(128 * g);  // issues this warpgroup's TMA stores
      float* ex = reinterpret_cast<float*>(smem + F::OFF_EX);
      // The previous tile's TMA store of this warpgroup has finished reading its
      // staging rows (fin_bar orders this before the writes below).
      if (store_thread) bulk_wait_read0();
      if (ok) {
        if (nb_mine > 0) {
          ex[g * 256 + r] = m;
          ex[g * 256 + 128 + r] = l;
        }
        tc_fence_before();
        mbar_arrive(fin_bar);
        ok = mbar_wait(fin_bar, k & 1, abort_flag, p.err, kErrWaitOther);
      }
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      // The other warpgroup reads ex only before its o_free arrival, and this
      // warpgroup writes ex again only after a PV of the next tile, which waits for
      // o_free.
      const int nb_other = we.nblk - nb_mine;
      const float mo = nb_other > 0 ? ex[(g ^ 1) * 256 + r] : -INFINITY;
      const float lo_ = nb_other > 0 ? ex[(g ^ 1) * 256 + 128 + r] : 0.f;
      const int nb0 = g == 0 ? nb_mine : nb_other, nb1 = we.nblk - nb0;
      const float m0 = g == 0 ? m : mo, l0 = g == 0 ? l : lo_;
      const float m1 = g == 0 ? mo : m, l1 = g == 0 ? lo_ : l;
      float w0 = 1.f, w1 = 1.f, inv = 1.f;
      if (!SIGMOID) {
        const float M = fmaxf(m0, m1);
        w0 = (m0 == -INFINITY) ? 0.f : fast_exp2(m0 - M);
        w1 = (m1 == -INFINITY) ? 0.f : fast_exp2(m1 - M);
        const float L = l0 * w0 + l1 * w1;
        inv = L > 0.f ? 1.f / L : 0.f;
      }
      w0 *= inv;
      w1 *= inv;
      // 32 columns of both accumulators at a time, packed to bf16 pairs and written
      // to the staging half (full tiles: HD 128 as 128-byte rows in the 128-byte
      // swizzle, HD 64 as 64-byte rows unswizzled; one TMA store per warpgroup
      // follows) or straight to the output rows (a sequence's last, partial tile).
      uint8_t* out_half = smem + F::OFF_OUT + g * F::OUT_HALF;
      const bool staged = we.rows_here == kBQ;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + (size_t)(we.q_row0 + r) * p.ldo +
                            (size_t)we.h * HD + g * (HD / 2);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        const uint32_t col = (uint32_t)(g * (HD / 2) + 32 * c);
        // Both buffers are read unconditionally (allocated columns; conditional
        // loads cost spills): an accumulator that no block of the tile wrote holds
        // stale values, which the selects below discard.
        uint32_t oa[32], ob[32];
        tmem_ld32(tmem + lane_off + 256 + col, oa);
        tmem_ld32(tmem + lane_off + 256 + HD + col, ob);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float v0 = (nb0 > 0 ? __uint_as_float(oa[2 * e]) * w0 : 0.f) +
                           (nb1 > 0 ? __uint_as_float(ob[2 * e]) * w1 : 0.f);
          const float v1 = (nb0 > 0 ? __uint_as_float(oa[2 * e + 1]) * w0 : 0.f) +
                           (nb1 > 0 ? __uint_as_float(ob[2 * e + 1]) * w1 : 0.f);
          pk[e] = pack_bf16x2(v0, v1);
        }
        if (staged) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int cidx = 4 * c + q;
            const uint32_t off = HD == 128 ? (uint32_t)(r * 128 + ((cidx ^ (r & 7)) << 4))
                                           : (uint32_t)(r * 64 + (cidx << 4));
            st_shared_v4(out_half + off, pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
        } else if (r < we.rows_here) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st_global_v4(orow + 32 * c + 8 * q, pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      tc_fence_before();
      if (staged) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(o_free);  // the next tile's PVs may overwrite O
        if (staged) mbar_arrive(&stage_bar[g]);
      }
      if (staged) {
        if (store_thread) {
          if (!mbar_wait(&stage_bar[g], n_staged & 1, abort_flag, p.err, kErrWaitOther)) break;
          tma_store_2d(&tmO, out_half, we.h * HD + g * (HD / 2), we.q_row0);
          bulk_commit();
        }
        ++n_staged;
      }
      gb += we.nblk;
    }
    if (threadIdx.x == (unsigned)(128 * g)) bulk_wait0();  // this warpgroup's output stores are complete
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int HD, bool ALIBI, bool SIGMOID>
cudaError_t launch_variant(const CUtensorMap* maps, const FParams& p, int* ctr, int ntiles, int grid,
                           cudaStream_t s) {
  using F = PT<HD>;
  auto kern = attn_persist_kernel<HD, ALIBI, SIGMOID>;
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
  cudaError_t e = cudaMemsetAsync(ctr, 0, sizeof(int), s);  // the launch's tile counter
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, F::SMEM, s>>>(maps[0], maps[1], maps[2], maps[3], p, ctr, ntiles);
  return cudaGetLastError();
}

template <int HD> cudaError_t launch(const AttnArgs& a, cudaStream_t s) {
  alignas(64) CUtensorMap maps[4];
  const int rows = a.batch * a.seq;
  const int qd = a.num_heads * HD, kd = a.num_kv_heads * HD;
  const int BF16 = (int)CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, SW = (int)CU_TENSOR_MAP_SWIZZLE_128B;
  const int SWO = HD == 128 ? SW : (int)CU_TENSOR_MAP_SWIZZLE_NONE;  // the staging layout of the output
  if (!make_tma_2d(&maps[0], a.q, BF16, 2, qd, rows, a.ldq, 64, 128, SW) ||
      !make_tma_2d(&maps[1], a.k, BF16, 2, kd, rows, a.ldk, 64, 128, SW) ||
      !make_tma_2d(&maps[2], a.v, BF16, 2, kd, rows, a.ldk, 64, 128, SW) ||
      !make_tma_2d(&maps[3], a.out, BF16, 2, qd, rows, a.ldo, HD / 2, 128, SWO))
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
  const int64_t ntiles = (int64_t)p.nqt * a.num_heads * a.batch;
  if (ntiles >= INT_MAX / 2) return cudaErrorInvalidValue;
  const int grid = (int)std::min<int64_t>(ntiles, std::max(1, a.sm_count));
  const int nt = (int)ntiles;
  if (a.alibi)
    return a.sigmoid ? launch_variant<HD, true, true>(maps, p, a.tile_ctr, nt, grid, s)
                     : launch_variant<HD, true, false>(maps, p, a.tile_ctr, nt, grid, s);
  return a.sigmoid ? launch_variant<HD, false, true>(maps, p, a.tile_ctr, nt, grid, s)
                   : launch_variant<HD, false, false>(maps, p, a.tile_ctr, nt, grid, s);
}

}  // namespace

bool attn_persist_supported(const AttnArgs& a) { return a.tile_ctr != nullptr && attn_tc_supported(a); }

cudaError_t attn_prefill_persist(const AttnArgs& a, cudaStream_t s) {
  if (!attn_persist_supported(a)) return cudaErrorInvalidValue;
  return a.head_dim == 64 ? launch<64>(a, s) : launch<128>(a, s);
}

}  // namespace wv
