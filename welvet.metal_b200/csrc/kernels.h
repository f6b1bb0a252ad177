// Launch interfaces of the sm_100a kernels (host C++ side). Every launcher takes
// device pointers and a stream, allocates nothing, and returns a cudaError_t
// from the launch; asynchronous failures surface through the error word
// (`err`, device memory, one uint32) that every kernel writes on a bounded-wait
// timeout or an argument fault detected on the device.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wv {

// Error word values (device -> host).
enum : uint32_t {
  kErrNone = 0,
  kErrWaitFull = 1,   // MMA issuer waited too long for a TMA stage
  kErrWaitEmpty = 2,  // producer waited too long for a free stage
  kErrWaitAccFull = 3,
  kErrWaitAccEmpty = 4,
  kErrWaitOther = 5,
  kErrPeerWait = 6,   // a peer rank's data did not arrive (peer-memory all-reduce)
};

// --------------------------------------------------------------------- GEMM
// C[M,N] = A[M,K] * B[N,K]^T with FP32 accumulation in TMEM. A and B are
// row-major with K contiguous (the reference's W[out,in] layout,
// src/layers/dense/dense.cpp:118). Operand encodings:
enum GemmKind : int {
  kGemmBF16 = 0,   // A bf16, B bf16
  kGemmTF32x3 = 1, // A = a_hi + a_lo, B = b_hi + b_lo (FP32 arrays holding TF32 values);
                   // three TF32 products per k (hi*hi + hi*lo + lo*hi), ~FP32 accuracy
  kGemmFP8 = 2,    // A bf16, B FP8-E4M3 codes (+ one FP32 scale per B row, epilogue)
  kGemmNF4 = 3,    // A bf16, B NF4 codes two per byte (+ FP32 absmax per 64 codes)
  // FormatNone codes of the reference's own quantisers (src/weights/native_codec.cpp),
  // dequantised in shared memory inside the mainloop; b_scale [N] holds the
  // per-output-row scale, applied in the epilogue (the per-tensor scale of the
  // matrix each row belongs to):
  kGemmI8 = 4,     // A bf16, B Int8 codes (one byte each; weight = code * scale)
  kGemmI4 = 5,     // A bf16, B Int4 codes two per byte, low nibble first (weight = q * scale)
  kGemmFP4 = 6,    // A bf16, B FP4 (E2M1) codes two per byte (weight = level; b_scale may be null)
};

struct GemmArgs {
  int kind = kGemmBF16;
  int M = 0, N = 0, K = 0;
  const void* a = nullptr;  // bf16 [M,lda] or fp32 hi [M,lda]
  const void* a_lo = nullptr;
  int lda = 0;              // elements
  const void* b = nullptr;  // bf16 / fp32 hi / fp8 codes / nf4 packed, [N,ldb]
  const void* b_lo = nullptr;
  int ldb = 0;              // elements (codes for fp8; bytes*2 for nf4 = K)
  const float* b_scale = nullptr;  // fp8: [N]; nf4: [N, K/64]
  // epilogue
  void* out = nullptr;      // [M, ldo]
  int ldo = 0;
  int out_bf16 = 0;         // 1: bf16 output, 0: fp32
  float* out_hi = nullptr;  // optional TF32 split of the output (fp32 outputs only)
  float* out_lo = nullptr;
  int split_only = 0;       // with out_hi: write only the split, not out
  // RoPE fused on columns [0, rope_cols), heads of head_dim columns, pairs (i, i+hd/2)
  const float2* rope_tab = nullptr; // [max_pos, head_dim/2] (cos, sin)
  int rope_cols = 0;
  int head_dim = 0;
  int rope_max_pos = 0;
  const int* positions = nullptr;   // per output row; else (row % pos_mod) or row
  int pos_mod = 0;
  // KV-cache scatter of the K/V column ranges (decode): columns [kv_col0, kv_col0+2*kd)
  // go to page pools instead of `out` when kv_k != null.
  void* kv_k = nullptr;
  void* kv_v = nullptr;
  const int* kv_slot = nullptr;     // per row: destination row index in the pools
  int kv_col0 = 0, kv_dim = 0;
  // SwiGLU: the N = 2 * inter_p columns alternate 32 gate / 32 up columns; the
  // epilogue writes h = SiLU(gate) * up to column (n / 64) * 32 + (n % 32) of out
  int swiglu = 0;
  int swiglu_cols = 0;  // h columns written (>= the last chunk is clipped); 0: all
  uint32_t* err = nullptr;
  int sm_count = 148;
  // Split-K workspace (FP32, splitk_ws_floats floats): when given and the output
  // has few tiles (M <= 128 decode rows), the K range is split over the SMs and a
  // second kernel adds the partials in order and applies the epilogue.
  float* splitk_ws = nullptr;
  size_t splitk_ws_floats = 0;
};
// Launches gemm_tc makes for these arguments (2 with split-K), and the split-K
// workspace (floats) the arguments' shape would use, 0 when it is not split.
int gemm_tc_launches(const GemmArgs& a);
size_t gemm_tc_splitk_floats(const GemmArgs& a);

// 2-D TMA descriptor over a row-major [outer][inner] matrix with row stride
// ld_elems (cuTensorMapEncodeTiled through the runtime's driver entry point).
// dt is a CUtensorMapDataType, sw a CUtensorMapSwizzle (ints to keep cuda.h out).
bool make_tma_2d(void* map128, const void* base, int dt, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t ld_elems, uint32_t box_inner, uint32_t box_outer, int sw);

// True when the tensor-core GEMM supports these shapes (TMA alignment).
bool gemm_tc_supported(const GemmArgs& a);
cudaError_t gemm_tc(const GemmArgs& a, cudaStream_t stream);
// Few-row BF16 projection (decode steps, M <= 64): streams the weights once at HBM
// rate on m16n8k16 MMAs, K split over a cluster of CTAs and reduced through
// distributed shared memory; RoPE and the KV page scatter in the epilogue
// (gemv_decode.cu). Uses a, lda, b (ldb == K), M, N, K, out (bf16), ldo, the RoPE
// and KV fields, err, sm_count.
bool gemv_decode_supported(const GemmArgs& a);
cudaError_t gemv_decode(const GemmArgs& a, cudaStream_t stream);
// One-shot all-reduce (sum) of a small vector over NVLink peer memory (peer.cu):
// every rank's receive area (slot [parity][sender] of slot_bytes, then the flags
// [parity][sender][kPeerCtas] uint32) mapped into this process; epoch = the call
// number (from 1, the same on every rank), parity = epoch & 1. count * element size
// must be a multiple of 16 bytes and at most slot_bytes; in/out 16-byte aligned,
// out may equal in.
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerCtas = 32;
struct PeerArgs {
  const void* in = nullptr;
  void* out = nullptr;
  size_t count = 0;
  int bf16 = 1;
  int nranks = 0, rank = 0;
  void* areas[kPeerMaxRanks] = {};
  size_t slot_bytes = 0;
  size_t flags_off = 0;
  uint32_t epoch = 0;
  uint64_t wait_ns = 0;
  uint32_t* err = nullptr;
};
cudaError_t peer_allreduce(const PeerArgs& a, cudaStream_t s);
// Owner side of a copy-engine reduce-scatter (peer.cu): slots[q] (q != rank, slot_bytes
// apart) hold the peers' partial of this rank's count elements, flags[q] becomes
// epoch once slot q has arrived; own (this rank's partial) is overwritten by the sum
// over ranks in rank order.
struct PeerRsArgs {
  void* own = nullptr;
  const void* slots = nullptr;
  const uint32_t* flags = nullptr;
  size_t count = 0;
  size_t slot_bytes = 0;
  int bf16 = 1;
  int nranks = 0, rank = 0;
  uint32_t epoch = 0;
  uint64_t wait_ns = 0;
  uint32_t* err = nullptr;
};
cudaError_t peer_rs_sum(const PeerRsArgs& a, int grid, cudaStream_t s);
// One warp waits (bounded) until flags[q] == epoch for every sender q != rank
// (code kErrPeerWait in *err on expiry); the attention-output exchange's barrier
// before the output projection.
cudaError_t peer_flags_wait(const uint32_t* flags, int nranks, int rank, uint32_t epoch, uint64_t wait_ns,
                            uint32_t* err, cudaStream_t s);

// CUDA-core fallback for shapes the TMA path cannot address (FP32 and BF16
// operands only; same epilogue semantics, RoPE excluded).
cudaError_t gemm_simt(const GemmArgs& a, cudaStream_t stream);

// ----------------------------------------------------------------- codecs
// decode(encode(w)) of FormatNone dtype 0-33, elementwise, bit-exact to the
// reference scalar codecs. `stats` = [absmax, min, max] of w from stats_f32,
// needed when codec_needs_stats(dtype), else may be null.
bool codec_dtype_supported(int dtype);
bool codec_needs_stats(int dtype);
cudaError_t codec_roundtrip_f32(int dtype, const float* w, float* out, int64_t n,
                                const float* stats, cudaStream_t s);
// [absmax, min, max] of w into out3 (device); scratch holds 3072 floats.
cudaError_t stats_f32(const float* w, int64_t n, float* out3, float* scratch, cudaStream_t s);
// Encoders/decoders of the stored byte formats.
cudaError_t codec_encode(int dtype, const float* w, void* codes, int64_t n, const float* nf4_scale,
                         cudaStream_t s);
cudaError_t codec_decode(int dtype, const void* codes, float* out, int64_t n,
                         const float* nf4_scale, cudaStream_t s);
// absmax over n floats into *out (device), via a two-pass reduction using `scratch`
// (>= 1024 floats).
cudaError_t absmax_f32(const float* w, int64_t n, float* out, float* scratch, cudaStream_t s);
// Extension formats: per-row FP8 scale and block-64 NF4.
cudaError_t fp8_rowscale_encode(const float* w, int rows, int cols, uint8_t* codes, float* scales,
                                cudaStream_t s);
cudaError_t fp8_rowscale_decode(const uint8_t* codes, const float* scales, int rows, int cols,
                                void* out, int out_bf16, cudaStream_t s);
cudaError_t nf4_block_encode(const float* w, int64_t n, uint8_t* packed, float* absmax,
                             cudaStream_t s);
cudaError_t nf4_block_decode(const uint8_t* packed, const float* absmax, int64_t n, void* out,
                             int out_bf16, cudaStream_t s);
// FormatNone Int8 (dtype 9), Int4 (14) or FP4 (16) codes of the reference quantisers
// for the dequantising GEMM kinds kGemmI8 / kGemmI4 / kGemmFP4, the per-tensor
// scale written once per row (n / cols rows; 1 for FP4). stats = [absmax, min, max].
cudaError_t formatnone_codes_encode(int dtype, const float* w, int64_t n, int cols, const float* stats,
                                    uint8_t* codes, float* row_scale, cudaStream_t s);
// Rewrites E4M3 codes in place to codes with the same reference-decoded value that
// the hardware E4M3 conversion decodes identically (no subnormal codes, no 0x7f/0xff).
cudaError_t fp8_normalize(uint8_t* codes, int64_t n, cudaStream_t s);

// ------------------------------------------------------------- elementwise
cudaError_t split_tf32(const float* x, float* hi, float* lo, int64_t n, cudaStream_t s);
cudaError_t cast_f32_bf16(const float* x, void* y, int64_t n, cudaStream_t s);
cudaError_t cast_bf16_f32(const void* x, float* y, int64_t n, cudaStream_t s);
// (cos, sin) of pos / theta^(fl32(2i/hd)) in double, rounded to float.
cudaError_t rope_table(float2* tab, int max_pos, int head_dim, double theta, cudaStream_t s);
// In-place RoPE on a [M, ld] matrix, columns [0, cols), heads of head_dim.
cudaError_t rope_apply(void* x, int is_bf16, int64_t M, int ld, int cols, int head_dim,
                       const float2* tab, int max_pos, const int* positions, int pos_mod,
                       cudaStream_t s);
// Deterministic synthetic data: element i of stream `seed` (SplitMix64 counter).
// kind 0: uniform(-a, a); kind 1: normal(0, a) (Box-Muller, double).
cudaError_t fill_synthetic(void* dst, int is_bf16, int64_t n, uint64_t seed, uint64_t offset,
                           int kind, double a, cudaStream_t s);

// ---------------------------------------------------------------- attention
struct AttnArgs {
  // q [*, ldq], k/v [*, ldk] token-major rows; head h at columns [h*hd, (h+1)*hd).
  const void* q = nullptr;
  const void* k = nullptr;
  const void* v = nullptr;
  int ldq = 0, ldk = 0;
  void* out = nullptr;  // [*, ldo]
  int ldo = 0;
  int is_bf16 = 0;
  int batch = 0, seq = 0;          // sequences x queries per sequence
  int num_heads = 0, num_kv_heads = 0, head_dim = 0;
  int stream_mode = 0;             // 1: reference stream semantics (single stream, block ends)
  int mask = 1, window = 0, max_seq_len = 512, prefix_len = 0, window_causal = 1;
  int alibi = 0, sigmoid = 0;
  int head_base = 0, total_heads = 0;  // ALiBi slope uses the global head index
  float scale = 0.f;
  float* out_hi = nullptr;         // optional TF32 split of the output
  float* out_lo = nullptr;
  uint32_t* err = nullptr;
  int sm_count = 148;
  int pair = -1;                   // tensor-core kernel: 1 CTA pairs (M = 256 UMMAs), 0 single CTAs, -1 auto
  // Tile counter of the persistent tensor-core kernel (one device int, zeroed by
  // each launch on its stream; launches that share it must not overlap in time).
  // Null: one CTA per query tile.
  int* tile_ctr = nullptr;
  // FP32 3xTF32 kernel: q/k/v are the TF32 hi parts, these the FP32 remainders
  // (same row strides).
  const void* q_lo = nullptr;
  const void* k_lo = nullptr;
  const void* v_lo = nullptr;
};
bool attn_tc_supported(const AttnArgs& a);
bool attn_tc_pair_supported(const AttnArgs& a);
cudaError_t attn_prefill_tc(const AttnArgs& a, cudaStream_t s);
// Persistent form of the BF16 tensor-core kernel (attn_persist.cu): needs tile_ctr.
bool attn_persist_supported(const AttnArgs& a);
cudaError_t attn_prefill_persist(const AttnArgs& a, cudaStream_t s);
cudaError_t attn_prefill_simt(const AttnArgs& a, cudaStream_t s);
// FP32 on the tensor cores (attn_tf32.cu): 3xTF32 flash attention, head_dim 64, no
// ring wrap; needs the hi / lo split of Q, K and V.
bool attn_tf32_supported(const AttnArgs& a);
cudaError_t attn_prefill_tf32(const AttnArgs& a, cudaStream_t s);
// FP32, head_dim 64/128, no ring wrap: register-tiled CUDA-core kernel (attn_f32.cu).
bool attn_f32_supported(const AttnArgs& a);
cudaError_t attn_prefill_f32(const AttnArgs& a, cudaStream_t s);

// Split-KV decode over a paged cache. Pools hold pages of kPageTokens rows of
// kd values (K and V separately, bf16 or fp32); block_table[b, j] names the
// page of tokens [16j, 16j+16) of sequence b. ctx_len[b] = tokens in the cache
// INCLUDING the new one (already appended).
constexpr int kPageTokens = 16;
struct DecodeArgs {
  const void* q = nullptr;  // [B, ldq] (after RoPE)
  int ldq = 0;
  const void* k_pool = nullptr;
  const void* v_pool = nullptr;
  const int* block_table = nullptr;
  int max_pages = 0;        // row stride of block_table
  const int* ctx_len = nullptr;
  void* out = nullptr;      // [B, ldo]
  int ldo = 0;
  int is_bf16 = 1;
  int batch = 0, num_heads = 0, num_kv_heads = 0, head_dim = 0;
  int alibi = 0, sigmoid = 0;
  int head_base = 0, total_heads = 0;  // ALiBi slope uses the global head index
  float scale = 0.f;
  int splits = 0;           // KV splits per (b, kv head); 0 = choose
  int max_ctx = 0;          // upper bound of ctx_len (split sizing)
  float* partial = nullptr; // scratch: [B, NH, splits, head_dim + 2]
  uint32_t* err = nullptr;  // device error word (bounded waits); may be null
  int sm_count = 148;
  int64_t pool_rows = 0;    // rows of the pools (pages * kv_heads * 16); 0 = unknown
};
int decode_splits(const DecodeArgs& a);
size_t decode_scratch_floats(const DecodeArgs& a);
// BF16 decode with TMA page loads and m16n8k16 MMAs (decode_tc.cu) when supported,
// else the CUDA-core kernel; then the split combine.
cudaError_t attn_decode(const DecodeArgs& a, cudaStream_t s);
bool decode_tc_supported(const DecodeArgs& a);
int decode_tc_ctas_per_sm(int head_dim);  // resident decode_tc_kernel CTAs per SM
cudaError_t attn_decode_tc(const DecodeArgs& a, int splits, cudaStream_t s);
// Append rows of k/v (token-major [rows, ld]) into the page pools at slot[row].
// Pool layout: [page][kv_head][kPageTokens][head_dim]; slot = page*kPageTokens + row.
cudaError_t kv_append(const void* k, const void* v, int ld, int rows, int kd, int head_dim,
                      int is_bf16, const int* slot, void* k_pool, void* v_pool, cudaStream_t s);

// ---- transformer-block kernels (block.cu)
struct NormArgs {
  int64_t rows = 0;
  int dim = 0;
  double eps = 1e-6;
  const void* x = nullptr;     // [rows, dim] FP32, or BF16 when x_bf16
  int x_bf16 = 0;
  const float* gamma = nullptr;  // [dim] decoded weights
  const float* beta = nullptr;   // [dim] (LayerNorm)
  void* pre = nullptr;           // x-hat [rows, dim] (may be null)
  void* post = nullptr;          // [rows, dim]
  int out_bf16 = 0;
  int vec4 = 0;                  // set by norm_forward
};
cudaError_t norm_forward(const NormArgs& a, int layernorm, cudaStream_t s);

struct EmbedArgs {
  int64_t tokens = 0;
  int vocab = 0, emb = 0, in_last = 1, act = -1;
  const float* W = nullptr;  // [vocab, emb] decoded weights
  const float* x = nullptr;  // ids as floats, token t at x[t * in_last]
  void* out = nullptr;       // [tokens, emb] FP32 or BF16
  int out_bf16 = 0;
  int vec4 = 0;              // set by embedding_forward
};
cudaError_t embedding_forward(const EmbedArgs& a, cudaStream_t s);

cudaError_t swiglu_pack_gate_up(const float* gate, const float* up, float* out, int inter, int in,
                                int inter_p, int in_p, cudaStream_t s);
cudaError_t pad_cols(const float* src, float* dst, int64_t rows, int cols, int cols_p, cudaStream_t s);
// x [rows, cols] -> zero-padded [rows, cols_p]: TF32 hi/lo pairs (hi != null) or BF16 (b)
cudaError_t pad_operand(const void* x, int x_bf16, int64_t rows, int cols, int cols_p, float* hi,
                        float* lo, void* b, cudaStream_t s);

// ---- bounded-wait probe (wait_probe.cu): one mbarrier wait that runs out after
// limit_ns and records kErrWaitOther in err
cudaError_t wait_probe(uint32_t* err, uint64_t limit_ns, cudaStream_t s);

// ---- MHA NormalBP leaf (mha_bwd.cu)
struct BwdArgs {
  int B = 0, T = 0;
  int64_t M = 0;
  int nh = 0, nk = 0, hd = 0, qd = 0, kd = 0, msl = 0;
  int mask = 1, window = 0, window_causal = 1, prefix = 0;
  int rope = 0, alibi = 0, sigmoid = 0;
  double theta = 10000.0, scale = 1.0;
  int shift = 0;                    // 64 when every attention gradient is below 1e-20
  const float* qkv = nullptr;       // [M, ld_qkv]: q | k | v projections (no RoPE)
  int ld_qkv = 0;
  const float* grad_attn = nullptr; // [M, qd]
  double* ck = nullptr;             // [msl, kd] key ring (rotated)
  double* cv = nullptr;             // [msl, kd]
  double* qb = nullptr;             // [T, qd] the batch's rotated q rows
  double* gyb = nullptr;            // [T, qd] the batch's attention gradient rows (x 2^shift)
  double* gq = nullptr;             // [T, qd]
  double* gk = nullptr;             // [msl, kd] key-gradient ring (kept across batches)
  double* gv = nullptr;             // [msl, kd]
  double* scratch = nullptr;        // [T * nh, 2 * kvmax]
  double* part_q = nullptr;         // [kMaxSplit, T, qd] q-gradient partials
  double* part_kv = nullptr;        // [2 * kMaxSplit, msl, kd] value / key gradient partials
  int kvmax = 0;
  float* g_q = nullptr;             // outputs, rows of stride ld_g
  float* g_k = nullptr;
  float* g_v = nullptr;
  int ld_g = 0;
};
constexpr int kMaxSplit = 4;       // reduction splits of the attention backward
cudaError_t attn_backward(const BwdArgs& a, cudaStream_t s);
int attn_backward_launches(const BwdArgs& a);  // kernels attn_backward launches
// src [rows, cols] -> [cols, rows_p] transposed, as TF32 hi/lo pairs, zero rows past `rows`
cudaError_t transpose_split(const float* src, int64_t rows, int cols, int64_t rows_p, float* hi, float* lo,
                            cudaStream_t s);
int mse_grid(int64_t n);
// grad = fl32(2 (pred - target) / n); partial[mse_grid(n)] = sums of squared differences
cudaError_t mse_grad(const float* pred, const float* target, float* grad, double* partial, int64_t n,
                     cudaStream_t s);
cudaError_t sgd_f32(const float* w, const float* g, float* out, int64_t n, double lr, cudaStream_t s);

} // namespace wv
