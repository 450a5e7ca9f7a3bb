// Allocation-free split-KV MLA decode (C ABI).  The contract, the callers it
// serves and the rules on concurrency and zeroing are in mla_decode_noalloc.h.
//
// Same kernels as the torch op `mla_decode` (mla_decode.cu); only the home of
// the split partials differs: a static __device__ array instead of per-call
// allocations.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "launchers.h"
#include "mla_decode_noalloc.h"

namespace {

constexpr size_t kScratchBytes = AFD_MLA_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
constexpr int kLatent = 512, kRope = 64;

struct DeviceSlot {
  std::atomic<bool> ready{false};
  float* scratch = nullptr;
  int* status = nullptr;
  int sms = 0;
};
DeviceSlot g_slots[kMaxDevices];
std::mutex g_setup_mutex;
thread_local char g_error[384] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// Partial O [batch, splits, heads, 512] fp32, then (256-byte aligned) the
// log-sum-exp [batch, splits, heads] fp32.
size_t scratch_bytes(int batch, int heads, int splits) {
  if (splits <= 1) return 0;
  const size_t rows = (size_t)batch * splits * heads;
  return align256(rows * kLatent * sizeof(float)) + rows * sizeof(float);
}

}  // namespace

// The split scratch and the internal status word, one copy per device.
static __device__ __align__(256) float g_mla_noalloc_scratch[kScratchBytes / sizeof(float)];
static __device__ int g_mla_noalloc_status;

namespace {

// One-time set-up for the current device: resolve the static symbols' device
// addresses and opt the decode kernel into its shared memory.
int setup_device(int dev, DeviceSlot*& out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(AFD_NOALLOC_EINVAL, "device %d out of range [0, %d)", dev, kMaxDevices);
  DeviceSlot& s = g_slots[dev];
  out = &s;
  if (s.ready.load(std::memory_order_acquire)) return AFD_NOALLOC_OK;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (s.ready.load(std::memory_order_relaxed)) return AFD_NOALLOC_OK;
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.scratch), g_mla_noalloc_scratch);
  if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.status), g_mla_noalloc_status);
  if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
  e = cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
  e = mla_decode_prepare_device();
  if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "shared-memory opt-in: %s", cudaGetErrorString(e));
  s.ready.store(true, std::memory_order_release);
  return AFD_NOALLOC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// The automatic split count: the torch op's pick, lowered until the partials
// fit in the static scratch (1 = unsplit, which needs none).
int auto_splits(int batch, int heads, int max_seq_len, int sms) {
  int splits = mla_decode_num_splits(batch * (heads / 16), max_seq_len, sms);
  const size_t row = (size_t)kLatent * sizeof(float) + sizeof(float);
  const size_t max_rows = (kScratchBytes - 256) / row;
  const size_t per_split = (size_t)batch * heads;
  if (splits > 1 && (size_t)splits * per_split > max_rows) splits = (int)(max_rows / per_split);
  while (splits > 1 && scratch_bytes(batch, heads, splits) > kScratchBytes) --splits;
  return splits < 1 ? 1 : splits;
}

}  // namespace

extern "C" int afd_mla_decode_noalloc_pick_splits(int batch, int heads, int max_seq_len) {
  if (batch <= 0 || heads <= 0 || heads % 16 != 0 || max_seq_len <= 0) return 1;
  int dev = -1;
  int sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 1;
  return auto_splits(batch, heads, max_seq_len, sms);
}

extern "C" uint64_t afd_mla_decode_noalloc_scratch_bytes(int batch, int heads, int num_splits) {
  if (batch <= 0 || heads <= 0) return 0;
  return (uint64_t)scratch_bytes(batch, heads, num_splits);
}

extern "C" int afd_mla_decode_noalloc(const void* q_lat, int64_t lat_sb, int64_t lat_sh, const void* q_pe,
                                      int64_t pe_sb, int64_t pe_sh, void* out, int64_t out_sb, int64_t out_sh,
                                      const void* cache, int num_blocks, int block_size, const int32_t* block_table,
                                      int table_stride, int max_blocks_per_seq, const int32_t* seq_lens, int batch,
                                      int heads, int num_splits, float scale, void* stream, int* status) {
  if (batch < 0 || heads <= 0) return fail(AFD_NOALLOC_EINVAL, "batch %d / heads %d", batch, heads);
  if (batch == 0) return AFD_NOALLOC_OK;
  if (!q_lat || !q_pe || !out || !cache || !block_table || !seq_lens)
    return fail(AFD_NOALLOC_EINVAL, "null tensor pointer");
  if (heads % 16 != 0) return fail(AFD_NOALLOC_EINVAL, "heads must be a multiple of 16 (got %d)", heads);
  if (block_size <= 0 || block_size % 32 != 0)
    return fail(AFD_NOALLOC_EINVAL, "block size must be a positive multiple of 32 (got %d)", block_size);
  if (num_blocks <= 0 || table_stride <= 0 || max_blocks_per_seq <= 0 || max_blocks_per_seq > table_stride)
    return fail(AFD_NOALLOC_EINVAL, "cache / block-table sizes (%d blocks, stride %d, %d columns)", num_blocks,
                table_stride, max_blocks_per_seq);
  if (!aligned16(q_lat) || !aligned16(q_pe) || lat_sb % 8 || lat_sh % 8 || pe_sb % 8 || pe_sh % 8)
    return fail(AFD_NOALLOC_EINVAL, "q rows must be 16-byte aligned");
  if (!aligned16(cache)) return fail(AFD_NOALLOC_EINVAL, "cache base must be 16-byte aligned (TMA source)");
  if (!aligned4(out) || out_sb % 2 || out_sh % 2)
    return fail(AFD_NOALLOC_EINVAL, "out must be 4-byte aligned with even strides (bf16 pairs are stored)");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  DeviceSlot* slot = nullptr;
  if (int rc = setup_device(dev, slot)) return rc;

  int splits = num_splits;
  if (splits <= 0) splits = auto_splits(batch, heads, max_blocks_per_seq * block_size, slot->sms);
  const size_t need = scratch_bytes(batch, heads, splits);
  if (need > kScratchBytes)
    return fail(AFD_NOALLOC_ETOOBIG,
                "split partials need %zu bytes (batch %d x splits %d x heads %d), the static scratch holds %zu; "
                "lower num_splits or the batch",
                need, batch, splits, heads, kScratchBytes);
  float* po = nullptr;
  float* pl = nullptr;
  if (splits > 1) {
    po = slot->scratch;
    pl = slot->scratch + align256((size_t)batch * splits * heads * kLatent * sizeof(float)) / sizeof(float);
  }
  MlaQO qo{};
  qo.q_lat = static_cast<const __nv_bfloat16*>(q_lat);
  qo.lat_sb = lat_sb;
  qo.lat_sh = lat_sh;
  qo.q_pe = static_cast<const __nv_bfloat16*>(q_pe);
  qo.pe_sb = pe_sb;
  qo.pe_sh = pe_sh;
  qo.out = static_cast<__nv_bfloat16*>(out);
  qo.out_sb = out_sb;
  qo.out_sh = out_sh;
  e = launch_mla_decode(qo, cache, block_table, seq_lens, po, pl, status ? status : slot->status, batch, heads,
                        kLatent, kRope, block_size, num_blocks, table_stride, splits, scale,
                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "launch: %s", cudaGetErrorString(e));
  return AFD_NOALLOC_OK;
}

extern "C" int afd_mla_decode_noalloc_status(int* value, int reset) {
  if (!value) return fail(AFD_NOALLOC_EINVAL, "null value pointer");
  cudaError_t e = cudaMemcpyFromSymbol(value, g_mla_noalloc_status, sizeof(int));
  if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "read status: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_mla_noalloc_status, &zero, sizeof(int));
    if (e != cudaSuccess) return fail(AFD_NOALLOC_ECUDA, "reset status: %s", cudaGetErrorString(e));
  }
  return AFD_NOALLOC_OK;
}

extern "C" const char* afd_mla_decode_noalloc_last_error(void) { return g_error; }
