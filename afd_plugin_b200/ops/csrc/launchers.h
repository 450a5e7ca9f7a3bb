// Host-side launchers of the afd_b200 kernels (torch-free interface).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

enum AfdDType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

// ---- elementwise.cu
void launch_rms_norm(void* out, const void* x, const void* w, int rows, int hidden, float eps, int dtype,
                     cudaStream_t s);
void launch_fused_add_rms_norm(void* out, const void* x, void* residual, const void* w, int rows, int hidden,
                               float eps, int dtype, cudaStream_t s);
void launch_silu_and_mul(void* out, const void* in, int rows, int d, int dtype, cudaStream_t s);
void launch_rope(void* x, const int64_t* pos, const float* cos_sin, int tokens, int heads, int rot, int64_t st,
                 int64_t sh, bool interleaved, int dtype, cudaStream_t s);
void launch_topk_route(const float* logits, const float* bias, float* w, int32_t* ids, int tokens, int E, int k,
                       int scoring, bool renorm, int n_group, int topk_group, float scale, const int32_t* forced,
                       cudaStream_t s);
// q_pe (optional, [T, q_heads, R] with strides q_st / q_sh) is rotated in place
// by the same launch.
void launch_mla_cache_write(void* cache, const void* kv_a, const void* w, float eps, const int64_t* pos,
                            const float* cos_sin, const int64_t* slots, int tokens, int L, int R, int64_t kv_stride,
                            int dtype, cudaStream_t s, void* q_pe = nullptr, int q_heads = 0, int64_t q_st = 0,
                            int64_t q_sh = 0);
// GQA prologue (see elementwise.cu): q / k RMSNorm when qw / kw are given,
// NeoX RoPE on whole heads, q -> q_out [T, nq, d], k / v -> caches [slots,
// nkv, d].  Returns false (nothing launched) for a head size it does not take
// (d = 32, 64, 128 or 256).
bool launch_gqa_prologue(const void* qkv, int64_t qkv_stride, int tokens, int nq, int nkv, int d, const void* qw,
                         const void* kw, float eps, const int64_t* pos, const float* cos_sin, void* q_out, void* kc,
                         void* vc, const int64_t* slots, int dtype, cudaStream_t s);
void launch_gqa_cache_write(void* kc, void* vc, const void* k, const void* v, const int64_t* slots, int tokens,
                            int row_elems, int64_t k_stride, int64_t v_stride, int dtype, cudaStream_t s);

// out[r] = argmax over row r of x [rows, n] (row stride ld elements; lowest index on ties).
void launch_argmax_rows(const void* x, int64_t ld, int rows, int n, int dtype, int32_t* out, cudaStream_t s);
// out[c * span + r] = sigmoid(x[r] . w), x [rows, H] bf16 (H % 8 == 0), w [H] bf16, c < copies.
void launch_gate_sigmoid_rows(const void* x, const void* w, int rows, int H, float* out, int copies, int span,
                              cudaStream_t s);

void launch_decode_advance(int32_t* input_ids, int64_t* positions, int64_t* slots, int32_t* seq_lens,
                           const int32_t* next_tokens, const int32_t* table, int batch, int table_stride,
                           int block_size, int64_t wrap_at, int64_t wrap_to, cudaStream_t s);

// ---- mla_decode.cu
// q [B, H, D] bf16 (D = L + R), cache [nblocks, bs, D] bf16, out [B, H, L] bf16.
// Scratch (num_splits > 1): partial_o [B, splits, H, L] fp32, partial_lse [B, splits, H] fp32.
// status: device int, set non-zero if a pipeline wait gave up.
// Query halves and output addressed through element strides (batch, head):
// the latent query and output may be head-major ([H, B, 512]) so the
// absorbed up-projections run as plain batched GEMMs without copies.
struct MlaQO {
  const __nv_bfloat16* q_lat;
  int64_t lat_sb, lat_sh;
  const __nv_bfloat16* q_pe;
  int64_t pe_sb, pe_sh;
  __nv_bfloat16* out;
  int64_t out_sb, out_sh;
};
int mla_decode_num_splits(int batch, int max_seq_len, int num_sms);
cudaError_t mla_decode_prepare_device();
// Returns cudaSuccess after launching, or an error with nothing launched: the
// cache base is not 16-byte aligned (a TMA rule), the shared-memory opt-in
// failed, or the cache's tensor map could not be encoded.  With split
// partials, `arrivals` (batch x heads/16 int32, all zero; left zero) lets the
// last CTA of each group merge them in the same launch; nullptr launches the
// separate combine kernel.  Launches sharing `arrivals` must be stream-ordered.
cudaError_t launch_mla_decode(const MlaQO& qo, const void* cache, const int32_t* block_table,
                              const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status, int batch,
                              int heads, int L, int R, int block_size, int num_blocks, int max_blocks_per_seq,
                              int num_splits, float scale, cudaStream_t s, int* arrivals = nullptr);
// Work-balanced variant: `ctas` CTAs per 16-head group split the concatenated
// KV tiles of all requests evenly; partial_o [2 * ctas, heads, 512] and
// partial_lse [2 * ctas, heads] fp32; arrivals: >= batch * heads / 16 zeroed
// ints (left zero).  batch <= mla_decode_balanced_max_batch().  Returns
// cudaErrorNotSupported (nothing launched) for shapes it does not take.
int mla_decode_balanced_ctas(int heads, int num_sms);
int mla_decode_balanced_max_batch();
cudaError_t launch_mla_decode_balanced(const MlaQO& qo, const void* cache, const int32_t* block_table,
                                       const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status,
                                       int* arrivals, int batch, int heads, int block_size, int num_blocks,
                                       int max_blocks_per_seq, int ctas, float scale, cudaStream_t s);
// ---- mla_decode_tc.cu (tcgen05 version of the same decode; DeepSeek 512 + 64
// latent, block sizes that are multiples of 64, heads a multiple of 16).
// Heads per CTA for `heads` (0 = unsupported), the split count for a batch,
// and the largest split count its in-launch merge takes.  Returns cudaErrorNotSupported
// (nothing launched) for a shape it does not take; split partials need
// `arrivals` as in launch_mla_decode.
int mla_decode_tc_heads_per_cta(int heads);
int mla_decode_tc_num_splits(int batch, int heads, int max_seq_len, int num_sms);
int mla_decode_tc_max_splits(int heads_per_cta);
cudaError_t launch_mla_decode_tc(const MlaQO& qo, const void* cache, const int32_t* block_table,
                                 const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status, int batch,
                                 int heads, int block_size, int num_blocks, int max_blocks_per_seq, int num_splits,
                                 float scale, cudaStream_t s, int* arrivals);
// Sparse (DeepSeek sparse attention) decode over keep_pos [B, num_keep] int32
// (-1 or a position >= seq_lens[b] = unused entry); same outputs and scratch,
// with splits over the kept entries.
void launch_mla_decode_sparse(const MlaQO& qo, const void* cache, const int32_t* block_table, const int32_t* seq_lens,
                              const int32_t* keep_pos, int num_keep, float* partial_o, float* partial_lse, int* status,
                              int batch, int heads, int L, int block_size, int max_blocks_per_seq, int num_splits,
                              float scale, cudaStream_t s, int* arrivals = nullptr);

// ---- tp_allreduce.cu: one-shot all-reduce of x [rows, H] bf16 (in place)
// over peer memory.  slot_ptrs / flag_ptrs: device int64 arrays of every
// rank's slots base ([2][world][slot_elems] bf16) and flags base
// ([max_ctas][world] uint64) in the symmetric heap; local_* are this rank's.
struct TPAllReduceParams {
  __nv_bfloat16* x;
  int rows, H, rows_per_cta, world, rank;
  int64_t slot_elems;
  const int64_t* slot_ptrs;
  const int64_t* flag_ptrs;
  const __nv_bfloat16* local_slots;
  const uint64_t* local_flags;
  uint64_t* epoch;
  unsigned* done_ctr;
  int* status;
  int64_t timeout_ns;
};
int tp_allreduce_rows_per_cta(int rows, int max_ctas);
cudaError_t launch_tp_allreduce(const TPAllReduceParams& p, cudaStream_t s);

// ---- gqa_decode.cu
// q [B, hq, 128], caches [blocks, bs, hkv, 128], out [B, hq, 128] (bf16).
void launch_gqa_decode(void* out, const void* q, const void* kc, const void* vc, const int32_t* block_table,
                       const int32_t* seq_lens, float* partial_o, float* partial_lse, int* status, int batch, int hq,
                       int hkv, int d, int block_size, int num_blocks, int max_blocks_per_seq, int num_splits,
                       float scale, cudaStream_t s);
int gqa_decode_num_splits(int batch, int hkv, int max_seq_len, int num_sms);

// ---- moe.cu
// Routing bookkeeping for a grouped expert GEMM over experts [offset, offset+E_local).
void launch_moe_align(const int32_t* topk_ids, int tokens, int k, int n_shared, int e_local, int offset,
                      int32_t* expert_counts, int32_t* expert_offsets, int32_t* row_token, int32_t* row_slot,
                      int32_t* token_slot_row, int* total_rows, cudaStream_t s);
void launch_moe_gather(void* xs, const void* x, const int32_t* row_token, int rows_cap, int hidden,
                       const int* total_rows, int dtype, cudaStream_t s);
void launch_moe_combine(void* out, const void* ys, const float* topk_w, const int32_t* token_slot_row, int tokens,
                        int k, int k_routed, int hidden, const void* shared_out, int dtype, cudaStream_t s);

// ---- afd_fused.cu
// Per-rank protocol: a token crosses NVLink once per FFN rank that owns one of
// its experts (or is its home rank for the shared expert / dense MLP), and
// comes back as one pre-reduced row per such FFN rank.
struct DispatchParams {
  const void* attn_out;   // [T, H] bf16
  void* residual;         // [T, H] bf16, updated in place
  const void* norm_w;     // [H] bf16 (post-attention RMSNorm)
  float eps;
  const void* gate_w;     // [E, H] bf16
  const float* gate_bias; // [E] or null
  int E, k, scoring, n_group, topk_group;
  bool renorm;
  float scale;
  int T, H;
  int moe;         // route to experts (0 for dense layers)
  int has_shared;  // the home FFN rank also applies the shared expert / dense MLP
  int num_ffn, e_local, t_cap, attn_rank, home_f, layer;
  const int64_t* tok_ptrs;     // [F] token rows [A, t_cap, H] (stage base) on each FFN rank
  const int64_t* rid_ptrs;     // [F] int32 [A, t_cap, k] routed expert ids
  const int64_t* rwt_ptrs;     // [F] fp32 [A, t_cap, k] routing weights
  const int64_t* tcount_ptrs;  // [F] int32 [A] tokens per source
  const int64_t* flag_ptrs;    // [F] uint64 arrival counters [layers]
  const int64_t* scale_ptrs;   // [F] fp32 [A, t_cap, H / 128] row scales (e4m3 rows) or null (bf16 rows)
  int32_t* fmask;              // local [t_cap]: FFN ranks that answer token t
  unsigned* done_ctr;          // local CTA-completion counter of the send kernel
  unsigned* route_ctr;         // local [ceil(T / 16)] router completion counters (zero between uses)
  void* h;                     // local scratch [T, H] bf16: normalised rows
  float* logits;               // local scratch [T, E] fp32: router logits
  int prenorm;                 // 1: attn_out is already the FFN input (no residual add / norm)
  const int32_t* hash_table;   // [vocab, k] expert ids per token id (hash-routed layer) or null
  const int32_t* input_ids;    // [T] token ids (with hash_table)
  int* status;
};
// FFN side: received token rows -> per-expert contiguous segments (local copies).
struct ExpandParams {
  const void* tok;        // [A, t_cap, H] (stage base, local)
  const int32_t* rid;     // [A, t_cap, k]
  const float* rwt;       // [A, t_cap, k]
  const int32_t* tcount;  // [A]
  void* x;                // [e_local * cap, H] expert segments
  int32_t* meta;          // [e_local * cap] (src << 24 | token << 8 | slot)
  float* rw;              // [e_local * cap]
  const float* tok_scale; // [A, t_cap, H / 128] when the rows arrive as e4m3 (tok is then bytes), else null
  void* home_x;           // [ratio * t_cap, H] bf16 copies of the home sources' rows (e4m3 rows only)
  int32_t* counts;        // [e_local + n_chunks] (or [e_local + ratio] without shared chunks)
  int A, t_cap, k, H, e_local, e_offset, cap, ratio, home_a0, moe;
  // Shared experts as virtual experts: chunk c's rows are every home source's
  // tokens, stored at x[shared_base + c * shared_stride + home position].
  int n_chunks, shared_base, shared_stride;
  // Arrival wait folded into the kernel (flag == nullptr: no wait).
  const uint64_t* flag;
  const uint64_t* epoch;
  uint64_t arrivals;
  int64_t timeout_ns;
  int* status;
};
// FFN side: per (source, token) sum of this rank's expert outputs (+ shared),
// one row stored into the source Attention rank's combine slot for this rank.
struct CombineSendParams {
  const void* staging;    // [A, t_cap, J, H] weighted expert outputs (local); or token rows in echo mode
  const int32_t* rid;     // [A, t_cap, k]
  const float* rwt;       // [A, t_cap, k] (echo mode)
  const int32_t* tcount;  // [A]
  int A, t_cap, k, J, H, e_local, e_offset, ratio, home_a0, moe, has_shared, f_rank, num_ffn, layer;
  int echo;               // 1: transport-only stand-in (scale the token row by its local weights)
  const float* tok_scale; // echo with e4m3 rows: [A, t_cap, H / 128] scales (staging holds the e4m3 rows)
  int home_slots;         // shared-expert slots k .. k + home_slots - 1 filled for home sources
  const int64_t* dst_ptrs;   // [A] combine buffers [t_cap, F, H] (stage base)
  const int64_t* flag_ptrs;  // [A] combine counters [layers]
  unsigned* done_ctr;
};
struct CombineParams {
  void* out;              // [T, H] bf16
  const void* comb;       // [t_cap, F, H] bf16 (stage base, local)
  const int32_t* fmask;   // [t_cap]
  int T, H, F;
  const uint64_t* flag;   // [layers] (stage base, local)
  int layer;
  const uint64_t* epoch;
  uint64_t arrivals;
  int64_t timeout_ns;
  int* status;
};
void launch_afd_epoch(uint64_t* epoch, cudaStream_t s);
// buf[idx] = the device's global nanosecond timer once the stream gets there.
void launch_afd_stamp(uint64_t* buf, int idx, cudaStream_t s);
void launch_afd_wait(const uint64_t* flag, const uint64_t* epoch, uint64_t arrivals, int64_t timeout_ns, int* status,
                     cudaStream_t s);
void launch_afd_dispatch(const DispatchParams& p, cudaStream_t s);
void launch_afd_expand(const ExpandParams& p, cudaStream_t s);
void launch_afd_combine_send(const CombineSendParams& p, cudaStream_t s);
void launch_afd_combine(const CombineParams& p, cudaStream_t s);

// ---- gemm_tcgen05.cu
// Epilogue 2 ("scatter") stores routing-weighted rows straight into the
// originating Attention ranks' combine buffers and signals them when the last
// CTA of the layer is done.
struct ScatterParams {
  const int32_t* meta;      // [rows] (src << 24 | token << 8 | slot)
  const float* rw;          // [rows] routing weight
  const int64_t* dst_ptrs;  // [A] combine buffer (stage base) on each Attention rank
  int J, H;                 // slots per token, hidden size
  unsigned* done_ctr;       // local, counts CTAs of the layer's scatter launches
  int total_ctas;           // CTAs across all scatter launches of the layer
  const int64_t* flag_ptrs; // [A] uint64 combine counters (stage base)
  int num_dst, layer;
  int32_t* counts_reset;    // local counters cleared before signalling
  int n_reset;
};
// Grouped GEMM D[r, n] = sum_k A[r, k] * W[e(r), n, k] over row segments of
// experts (rows of expert e: [offsets[e], offsets[e] + counts[e])).
// epilogue: 0 = store bf16, 1 = SiLU(gate) * up over paired halves (N = 2I -> I).
// CTAs of a persistent grouped-GEMM launch over n_items (expert, tile) items.
int grouped_gemm_grid(int n_items);
// Same with block-scaled fp8 (e4m3) weights: w [E, N, K] bytes, w_scale
// [E, ceil(N / 128), K / 128] fp32 (128 x 128 blocks); bf16 activations.
// K % 128 == 0; epilogue 1 needs I % 64 == 0 and epilogue 0 / 2 N % 128 == 0.
void launch_grouped_gemm_w8(void* d, const void* a, const void* w, const float* w_scale, const int32_t* expert_offsets,
                            const int32_t* expert_counts, int e_local, int rows_cap, int n, int k, int epilogue,
                            int* status, cudaStream_t s, int w_experts, const ScatterParams* sp);
// w_expert_rows: rows between consecutive experts in W (0 = one weight set
// shared by every segment, e.g. shared experts / dense MLP over per-source segments).
// A pass covers up to 256 rows of an expert; wider segments take several
// passes over its weights.
void launch_grouped_gemm(void* d, const void* a, const void* w, const int32_t* expert_offsets,
                         const int32_t* expert_counts, int e_local, int rows_cap, int n, int k, int epilogue,
                         int* status, cudaStream_t s, int w_experts = -1, const ScatterParams* sp = nullptr);

// One grouped GEMM of a launch (bf16 weights).
//   epilogue 0: d[r, n] (row-major [rows_cap, N]); 1: SwiGLU over paired halves
//   (d [rows_cap, N / 2]); 2: routing-weighted scatter (ScatterParams);
//   3: expert-blocked columns, d[r - offsets[e], e * N + n] (d [rows, e_local * N]),
//   e.g. a per-head batched product written token-major for the next GEMM.
struct GemmSpec {
  void* d;                 // output (see above); unused for epilogue 2
  const void* a;           // activations: rows of K elements, a_ld apart
  const void* w;           // weights [w_experts, N, K]
  const int32_t* offsets;  // [e_local] first row of each expert's segment
  const int32_t* counts;   // [e_local] rows of each expert
  int e_local, rows_cap, n, k, epilogue;
  int w_experts;           // -1: e_local; 1: one weight set for every segment
  int fixed_count = 0;     // with counts == nullptr: every segment has this many rows, starting at row 0
  int k_splits = 1;        // > 1 (epilogue 0 / 3): K is split over that many items per tile; each adds its fp32
                           // partial into acc_ws and the last one to finish a tile writes d and re-zeroes acc_ws
  float* acc_ws = nullptr; // [rows_cap, output columns] fp32, zero between launches
  int* tile_ctr = nullptr; // [e_local * n_tiles] int32, zero between launches
  int out_f32 = 0;         // epilogue 0: d is float (fp32 results)
  int n_valid = 0;         // epilogue 0: store only columns < n_valid (0: all N); the output's row stride is
                           // then n_valid (weights padded to a multiple of 128 rows)
  int64_t a_ld = 0;        // elements between activation rows (0: K)
  int64_t a_plane = 0;     // > 0: expert e's rows start a_plane * e elements in (a 3-D view); offsets are then
                           // rows within the expert's plane
};
// Kernel-side description of a phase (filled by the launcher).
struct GGPhase {
  __nv_bfloat16* d;
  const int32_t* offsets;
  const int32_t* counts;
  int* done;  // phase 0 of a two-phase launch: finished tiles per expert (zero between launches)
  int n_w, w_stride_rows, k_dim, ld_d, n_tiles, n_experts, epi;
  int a3d;    // activation tiles from a 3-D tensor map (k, row, expert)
  int fixed_count;  // counts == nullptr: rows per segment (segments start at row 0)
  int out_f32;      // epilogue 0: fp32 output
  int n_valid;      // epilogue 0: columns stored
  int k_splits;     // items per tile along K
  int kb_per;       // K blocks per split
  float* acc_ws;    // split-K fp32 partial sums [rows, ld_d]
  int* tile_ctr;    // split-K arrivals per (expert, tile)
};
struct GGArgs {
  GGPhase ph[2];
  int n_phases;
  int* status;
  unsigned* finish_ctr;    // two-phase launches: CTAs done (zero between launches)
  long long dep_timeout_ns;
  int l2_hints;            // L2 eviction policies on the weight stream (0 = plain loads)
};
// One launch of one or two grouped GEMMs.  With g1, phase 1 reads phase 0's
// output (its `a` is g0's `d`, same row segments): an MoE layer's gate_up
// (epilogue 1) and down projection (epilogue 0 or 2) in one persistent
// kernel.  done: int32 [g0.e_local] and finish_ctr: one uint32, both zero
// before the first launch and left zero by every launch.  rows_hint: the
// largest row count expected in one segment; it picks the tokens per pass
// (and so the pipeline depth), never the result.  Returns the launch error.
cudaError_t launch_grouped_gemm_phases(const GemmSpec& g0, const GemmSpec* g1, int* done, unsigned* finish_ctr,
                                       int* status, const ScatterParams* sp, cudaStream_t s, int rows_hint = 512);

// ---- gdn.cu (Gated DeltaNet)
struct GdnConvParams {
  const __nv_bfloat16* x;  // [T, >= C], row stride ldx (q | k | v channels first)
  int64_t ldx;
  const __nv_bfloat16* weight;  // [C, K]
  __nv_bfloat16* state;         // [slots, C, K - 1] last K - 1 inputs, oldest first
  __nv_bfloat16* y;             // [T, C]
  const int32_t* cu_seqlens;    // [S + 1]
  const int32_t* slots;         // [S]
  const int32_t* reset;         // [S] or null
  int num_seqs, C, K;
};
struct GdnRecurrentParams {
  const __nv_bfloat16* qkv;  // [T, 2 * nk * dk + nv * dv] (q | k | v), row stride ld_qkv
  int64_t ld_qkv;
  const __nv_bfloat16* z;    // [T, nv * dv] gate, row stride ld_z
  int64_t ld_z;
  const __nv_bfloat16* a;    // [T, nv] (decay input), row stride ld_ab
  const __nv_bfloat16* b;    // [T, nv] (beta input)
  int64_t ld_ab;
  const float* A_log;        // [nv]
  const float* dt_bias;      // [nv]
  const __nv_bfloat16* norm_w;  // [dv]
  float eps;
  float* state;              // [slots, nv, dk, dv]
  __nv_bfloat16* out;        // [T, nv * dv]
  const int32_t* cu_seqlens;
  const int32_t* slots;
  const int32_t* reset;
  int num_seqs, nk, nv, dk, dv;
};
void launch_gdn_conv(const GdnConvParams& p, cudaStream_t s);
bool launch_gdn_recurrent(const GdnRecurrentParams& p, cudaStream_t s);
