// Allocation-free C entry point for split-KV MLA decode.
//
// No counterpart in the reference: the reference runs attention through its
// serving framework's own kernels and has no C entry point of its own.  This
// one exists for callers that may not allocate device memory during a call:
//   * a C/C++ serving runtime that carves all device memory into fixed arenas
//     at start-up (weights, KV cache) and forbids growth afterwards, so a
//     caching allocator cannot be used for per-call scratch;
//   * code on a latency-critical path, where cudaMalloc / cudaFree can
//     synchronise the device and stall every stream;
//   * a host process that does not run PyTorch at all, so there is no caching
//     allocator to draw from.
//
// The split-KV partials (normalised O and log-sum-exp per split) live in one
// file-scope static __device__ array of AFD_MLA_NOALLOC_SCRATCH_BYTES bytes,
// reserved per device when the module is loaded.  The call itself performs no
// cudaMalloc / cudaFree and calls no allocating library.
//
// Rules for callers:
//   * Make the device that holds the tensors current before the call.
//   * The first call on a device runs a one-time set-up (symbol lookup, which
//     loads the module, and the kernel's shared-memory opt-in).  Make that
//     first call before any stream capture, e.g. with a small warm-up call.
//   * Calls on one device share the one scratch array.  Two calls in flight
//     at the same time on one device (different streams, or different host
//     threads without ordering) race on it and corrupt each other's output.
//     Serialise them: one stream, or order the streams with events.
//   * Nothing in the scratch has to start at zero: every partial that the merge
//     step reads is written earlier in the same call.  The status word
//     (`status`, or the internal one) must read zero before a call for a
//     non-zero value afterwards to mean that this call timed out.
//   * With num_splits <= 0 the split count is picked automatically and always
//     fits: the pick is lowered until the partials fit in the scratch (down to
//     one split, which needs none).  afd_mla_decode_noalloc_pick_splits says
//     which count a call will use.  An explicit num_splits whose partials would
//     not fit is rejected with AFD_NOALLOC_ETOOBIG and nothing is launched.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AFD_MLA_NOALLOC_SCRATCH_BYTES (16u << 20)  // 16 MiB per device

enum {
  AFD_NOALLOC_OK = 0,
  AFD_NOALLOC_EINVAL = 1,   // bad argument (null pointer, shape, alignment)
  AFD_NOALLOC_ETOOBIG = 2,  // split partials exceed the static scratch
  AFD_NOALLOC_ECUDA = 3,    // a CUDA runtime call failed
};

// q_lat [batch, heads, 512] and q_pe [batch, heads, 64]: bf16, last dimension
// contiguous, row strides (in elements) multiples of 8, 16-byte aligned bases.
// out: bf16, element (b, h, c) at out + b * out_sb + h * out_sh + c; the base
// 4-byte aligned and out_sb, out_sh even (pairs of bf16 are stored together).
// cache [num_blocks, block_size, 576] bf16 contiguous, base 16-byte aligned
// (the kernel reads it with TMA); block_table int32 with
// `table_stride` elements between rows and `max_blocks_per_seq` used columns;
// seq_lens int32 [batch].  heads % 16 == 0, block_size % 32 == 0.
// num_splits <= 0 picks the split count from the batch, the context length
// and the SM count, capped so the partials fit in the scratch.
// status: device int that records a pipeline wait timeout, or NULL for the
// internal per-device word (read it with afd_mla_decode_noalloc_status).
// stream: a cudaStream_t (NULL = legacy default stream).
int afd_mla_decode_noalloc(const void* q_lat, int64_t lat_sb, int64_t lat_sh, const void* q_pe, int64_t pe_sb,
                           int64_t pe_sh, void* out, int64_t out_sb, int64_t out_sh, const void* cache, int num_blocks,
                           int block_size, const int32_t* block_table, int table_stride, int max_blocks_per_seq,
                           const int32_t* seq_lens, int batch, int heads, int num_splits, float scale, void* stream,
                           int* status);

// The split count a call with num_splits <= 0 uses on the current device for
// this batch, head count and longest context (max_blocks_per_seq * block_size).
int afd_mla_decode_noalloc_pick_splits(int batch, int heads, int max_seq_len);

// Scratch bytes a call with these sizes needs (0 when it runs unsplit).
uint64_t afd_mla_decode_noalloc_scratch_bytes(int batch, int heads, int num_splits);

// Reads (and with reset != 0 clears) the internal status word of the current
// device.  Synchronous copy; not for use inside stream capture.
int afd_mla_decode_noalloc_status(int* value, int reset);

// Message of the calling thread's most recent failed call.
const char* afd_mla_decode_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
