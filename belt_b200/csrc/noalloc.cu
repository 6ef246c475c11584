// belt_latent_decode_noalloc: one decode step of a compressed layer (schedule -> split-KV decode -> merge) whose
// working memory is a fixed array inside this library, for callers that cannot allocate device memory.
//
// Who cannot allocate: a host that binds this library over its C ABI (ctypes, cgo, JNI, a C++ engine) and holds only
// the buffers its engine handed it -- the KV pool, the query and the output -- with no device allocator of its own to
// call; and serving engines that reserve nearly all of HBM for the KV pool at start-up, where a per-step cudaMalloc
// can fail, or stall the step while the driver maps memory. The regular entry points take the split-KV scratch
// (`work`, `cta_seg`, `seg_base`, `part`) from the caller; this one keeps it in `g_decode_scratch` below.
//
// The array holds kScratchBytes (24 MiB) on every GPU that loads the library, from the load until the process exits.
// Limits that follow from it, checked before anything runs: num_reqs <= kMaxReqs, num_ctas <= kMaxCtas, and
// (num_reqs + num_ctas) * 24 * (lv + 1) * 4 bytes of partials <= kPartBytes (at lv = 640 and 148 CTAs: 258 requests).
//
// Every call on a device uses the same array and leaves its contents there for the next call. No byte of it has to
// start at zero: the schedule writes every segment record, CTA range and request range that the decode and the merge
// of the same call read, and the decode writes every partial the merge reads. Calls whose work overlaps on the GPU
// (different streams of one device without an ordering between them, or several host threads on one device) race on
// the array and give wrong results; calls on one stream run one after the other.
//
// The split is the cost-weighted one (belt_decode_schedule_weighted) with the backend's start cost kStartCost: same
// outputs as the reference's equal-tiles split within the decode's tolerance, and less decode time. The backend also
// deals the cost out by measured CTA speed (belt_decode_schedule_balanced), which needs per-CTA times and weights kept
// from step to step; this entry keeps no state between calls, so it uses the weighted split alone.
//
// Where the array is: its device address belongs to the CUDA context that loaded this library's device code. Every
// call made outside stream capture looks it up again (cudaGetSymbolAddress, which can make the runtime load the
// device code in that context) and records it for the current context; a call made while `stream` is capturing uses
// the record of the current context and is refused if there is none. So the first call in a context (the first on a
// device, the first under a driver-API context a host made current, and the first after a cudaDeviceReset, which
// loads the device code again, possibly at another address) must come before any stream capture begins.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/belt_b200.h"
#include "common.cuh"
#include "launch.h"
#include "scratch_cache.h"

// The host-side name stands for the array; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_decode_scratch[24u << 20];

namespace {

constexpr size_t kScratchBytes = sizeof(g_decode_scratch);
constexpr int kMaxReqs = 4096;
constexpr int kMaxCtas = 1024;
constexpr int kStartCost = 13;     // the backend's start cost (extra cost of a request's first tile, eighths of a tile)
constexpr int kCacheSlots = 64;    // contexts remembered (oldest dropped beyond this)
// Schedule records at fixed offsets, then the partials.
constexpr size_t kWorkOff = 0;                                                   // [(kMaxReqs + kMaxCtas), 4] int32
constexpr size_t kCtaSegOff = kWorkOff + size_t(kMaxReqs + kMaxCtas) * 4 * 4;    // [kMaxCtas + 1] int32
constexpr size_t kSegBaseOff = (kCtaSegOff + size_t(kMaxCtas + 1) * 4 + 255) / 256 * 256;   // [kMaxReqs + 1] int32
constexpr size_t kPartOff = 128u << 10;
constexpr size_t kPartBytes = kScratchBytes - kPartOff;
static_assert(kSegBaseOff + size_t(kMaxReqs + 1) * 4 <= kPartOff, "schedule records overlap the partials");

std::mutex g_mu;
belt::ScratchAddressCache<kCacheSlots> g_scratch;

// Records the failure for belt_last_error() and returns `code`.
int reject(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int reject(int code, const char* fmt, ...) {
  char buf[768];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  belt::set_last_error(buf);
  return code;
}

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The calling thread's current driver context (the runtime's primary context of the current device, or a context a
// driver-API host made current), through the driver entry point the runtime exposes (no link against libcuda).
int current_context(CUcontext* ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return reject(BELT_ERR_CUDA, "latent_decode_noalloc: cuCtxGetCurrent is unavailable");
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  if (fn(ctx) != CUDA_SUCCESS || !*ctx) return reject(BELT_ERR_CUDA, "latent_decode_noalloc: no current CUDA context");
  return BELT_OK;
}

// Device address of the scratch array in the current context: looked up again outside stream capture, taken from the
// record of this context while `stream` captures.
int scratch_in_current_context(cudaStream_t stream, unsigned char** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return reject(BELT_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  const bool capturing = cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lock(g_mu);
  void* ptr = nullptr;
  CUcontext ctx = nullptr;
  if (capturing) {
    const int r = current_context(&ctx);
    if (r != BELT_OK) return r;
    ptr = g_scratch.find(ctx);
    if (!ptr)
      return reject(BELT_ERR_INVALID,
                    "latent_decode_noalloc: first call in this CUDA context (device %d) made during stream capture; "
                    "make one call outside capture first", dev);
  } else {
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess)
      return reject(BELT_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s (%s)", dev, cudaGetErrorString(e),
                    cudaGetErrorName(e));
    if (!ptr || (reinterpret_cast<uintptr_t>(ptr) & 255u))
      return reject(BELT_ERR_CUDA, "scratch array on device %d is not 256-byte aligned", dev);
    // the lookup made the context current if it was not yet (the runtime's primary context of `dev`)
    const int r = current_context(&ctx);
    if (r != BELT_OK) return r;
    g_scratch.refresh(ctx, ptr);
  }
  *out = static_cast<unsigned char*>(ptr);
  return BELT_OK;
}

// The failure text of a regular entry point this one called.
int forward(int status, const char* step) {
  return reject(status, "%s: %s", step, belt_last_error());
}

}  // namespace

extern "C" {

int belt_latent_decode_noalloc(const void* q_bd, int32_t num_reqs, int32_t kq, const void* cache, int64_t num_blocks,
                               int32_t page, int32_t row_width, int64_t stride_block, int64_t stride_tok,
                               const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                               int32_t num_ctas, int32_t min_tiles, float sm_scale, int32_t lk_pad, int32_t lv,
                               const int32_t* rope_groups, const void* rope_blocks, int32_t n_rope_blocks,
                               const void* cos_sin, int32_t max_pos, void* out, int64_t out_sb, int64_t out_sh,
                               float* lse, int64_t lse_sb, int32_t* err, void* stream) {
  if (num_reqs < 0 || num_reqs > kMaxReqs)
    return reject(BELT_ERR_INVALID, "latent_decode_noalloc: num_reqs %d outside [0, %d] (fixed scratch)", num_reqs,
                  kMaxReqs);
  if (num_ctas < 1 || num_ctas > kMaxCtas)
    return reject(BELT_ERR_INVALID, "latent_decode_noalloc: num_ctas %d outside [1, %d] (fixed scratch)", num_ctas,
                  kMaxCtas);
  if (lv <= 0 || lv > 640) return reject(BELT_ERR_INVALID, "latent_decode_noalloc: lv %d outside (0, 640]", lv);
  const long long part_sh = lv + 1, part_ss = 24 * part_sh;
  const long long need = (static_cast<long long>(num_reqs) + num_ctas) * part_ss * 4;
  if (need > static_cast<long long>(kPartBytes))
    return reject(BELT_ERR_INVALID,
                  "latent_decode_noalloc: (num_reqs %d + num_ctas %d) segments x 24 heads x (lv %d + 1) fp32 = %lld "
                  "bytes of partials exceed the fixed scratch of %lld bytes",
                  num_reqs, num_ctas, lv, need, static_cast<long long>(kPartBytes));
  if (num_reqs == 0) {
    belt::set_last_error("");
    return BELT_OK;
  }
  if (!out || !lse || !seq_lens) return reject(BELT_ERR_INVALID, "latent_decode_noalloc: null buffer");

  unsigned char* base = nullptr;
  int r = scratch_in_current_context(reinterpret_cast<cudaStream_t>(stream), &base);
  if (r != BELT_OK) return r;
  int32_t* work = reinterpret_cast<int32_t*>(base + kWorkOff);
  int32_t* cta_seg = reinterpret_cast<int32_t*>(base + kCtaSegOff);
  int32_t* seg_base = reinterpret_cast<int32_t*>(base + kSegBaseOff);
  float* part = reinterpret_cast<float*>(base + kPartOff);

  r = belt_decode_schedule_weighted(seq_lens, num_reqs, num_ctas, min_tiles, kStartCost, work,
                                    static_cast<int64_t>(num_reqs) + num_ctas, cta_seg, seg_base, err, stream);
  if (r != BELT_OK) return forward(r, "latent_decode_noalloc");
  r = belt_latent_decode(q_bd, num_reqs, kq, cache, num_blocks, page, row_width, stride_block, stride_tok, block_table,
                         bt_stride, seq_lens, work, cta_seg, num_ctas, part, part_ss, part_sh, sm_scale, lk_pad, lv,
                         rope_groups, rope_blocks, n_rope_blocks, cos_sin, max_pos, err, stream);
  if (r != BELT_OK) return forward(r, "latent_decode_noalloc");
  r = belt_merge_segments(part, part_ss, part_sh, seg_base, num_reqs, 24, lv, out, out_sb, out_sh, lse, lse_sb,
                          stream);
  if (r != BELT_OK) return forward(r, "latent_decode_noalloc");
  belt::set_last_error("");
  return BELT_OK;
}

}  // extern "C"
