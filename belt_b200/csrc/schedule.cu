// Split-KV work schedule of one decode step, computed on the device (graph-safe: fixed grid, persistent buffers).
//
// With unit 1 and start cost 0 this is the reference's ``_schedule`` split (plugins/vllm_lrkv/vllm_lrkv/
// cute_decode.py:571-607): every request's context is cut into `tile`-token tiles, the tiles of the whole batch
// (request order) are dealt out in equal runs of per = max(ceil(total / num_ctas), min_tiles, 1) tiles to the CTAs,
// and a run that crosses request boundaries becomes several segments. The weighted split (unit 8, start cost s) deals
// out cost instead: a tile costs 8 units and every request's first tile s more, so that a CTA which switches between
// requests (a query reload and a partial-output epilogue per switch) gets fewer tiles. In both:
//   work[k]     = (request, first tile, end tile, 0), segments in request order;
//   seg_base[b] = first segment of request b, seg_base[B] = number of segments;
//   cta_seg[c]  = first segment of CTA c, cta_seg[num_ctas] = number of segments.
// Balanced split (cta_w given): the CTAs' shares of the cost follow per-CTA speed weights learned from the decode
// launches' measured times (cta_ns / cta_cap of the previous step), so that CTAs on slower SMs get less work:
// CTA c covers the costs [B_c, B_(c+1)) with B_c = per * num_ctas * W_c / W (W_c the weights' prefix sum), which is
// c * per when every weight is equal.
// One CTA of 1024 threads; requests are processed in chunks of 1024 with block-wide exclusive scans.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int kSchedThreads = 1024;
constexpr int kMaxBalancedCtas = 1024;

// Block-wide exclusive scan of one value per thread; returns this thread's prefix and writes the total.
__device__ long long block_exclusive_scan(long long v, long long* warp_sums, long long* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  long long x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[w] = x;
  __syncthreads();
  if (w == 0) {
    long long s = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_sums[lane] = s;   // inclusive over warps
    if (lane == 31) *total = s;
  }
  __syncthreads();
  const long long before = (w > 0 ? warp_sums[w - 1] : 0) + x - v;
  __syncthreads();
  return before;
}
}  // namespace

__global__ void __launch_bounds__(kSchedThreads) schedule_kernel(const ScheduleParams p) {
  __shared__ long long warp_sums[32];
  __shared__ long long total_s;
  __shared__ long long bounds[kMaxBalancedCtas + 1];   // balanced split: first cost of every CTA
  const int B = p.num_reqs;
  const int tile = p.tile;
  const long long u = p.unit, s0 = p.start_cost;
  // pass 1: cost offset of every request (kept in seg_base until pass 2 overwrites it) and the total cost
  long long carry = 0;
  for (int b0 = 0; b0 < B; b0 += kSchedThreads) {
    const int b = b0 + threadIdx.x;
    const long long tiles = b < B ? (static_cast<long long>(p.seq_lens[b]) + tile - 1) / tile : 0;
    const long long cost = tiles > 0 ? s0 + u * tiles : 0;
    const long long ex = block_exclusive_scan(cost, warp_sums, &total_s);
    if (b < B) p.seg_base[b] = static_cast<int32_t>(carry + ex);
    carry += total_s;
    __syncthreads();
  }
  const long long total_cost = carry;
  long long per = (total_cost + p.num_ctas - 1) / p.num_ctas;
  per = per > u * p.min_tiles ? per : u * p.min_tiles;
  per = per > u ? per : u;
  auto cdiv = [](long long a, long long b) { return a >= 0 ? (a + b - 1) / b : -((-a) / b); };
  // balanced split: learn the weights from the previous step's times, then the CTAs' cost bounds
  const bool tuned = p.cta_w != nullptr;
  const bool balanced = tuned && per >= 8 * u && p.num_ctas <= kMaxBalancedCtas;
  if (tuned) {
    const int c = threadIdx.x;
    const bool mine = c < p.num_ctas;   // num_ctas <= 1024 whenever balanced
    float w = 1.f;
    double rate = 0.0;
    bool seen = true;
    if (balanced && mine) {
      w = p.cta_w[c];
      const long long ns = p.cta_ns[c], cap = p.cta_cap[c];
      seen = ns > 0 && cap > 0;
      rate = seen ? static_cast<double>(cap) / static_cast<double>(ns) : 0.0;
    }
    if (balanced && __syncthreads_and(seen ? 1 : 0)) {
      // mean rate over the CTAs (a fixed-point sum keeps the block scan integral and the result deterministic)
      const long long rq = mine ? static_cast<long long>(rate * 1e9) : 0;   // cost units per second
      block_exclusive_scan(rq, warp_sums, &total_s);
      const double mean = static_cast<double>(total_s) / p.num_ctas;
      if (mine && mean > 0.0) {
        const float r = static_cast<float>(static_cast<double>(rq) / mean);
        w = fminf(fmaxf(0.5f * w + 0.5f * r, 0.8f), 1.25f);
      }
    }
    if (balanced) {
      // normalise to mean 1 in fixed point (2^20 per unit weight), then the prefix sums give the bounds
      const long long wq = mine ? static_cast<long long>(w * 1048576.f + 0.5f) : 0;
      const long long before = block_exclusive_scan(wq, warp_sums, &total_s);
      const long long span = per * p.num_ctas, wsum = total_s;
      if (mine) {
        bounds[c] = span * before / wsum;
        p.cta_w[c] = static_cast<float>(static_cast<double>(wq) * p.num_ctas / static_cast<double>(wsum));
      }
      if (c == 0) bounds[p.num_ctas] = span;
      __syncthreads();
    }
    for (int k = threadIdx.x; k < p.num_ctas; k += kSchedThreads) {
      p.cta_cap[k] = balanced ? bounds[k + 1] - bounds[k] : per;
      p.cta_ns[k] = 0;
    }
  }
  // first cost of CTA c, and the CTA holding cost x (the last c with lo(c) <= x)
  auto lo = [&](long long c) -> long long { return balanced ? bounds[c] : c * per; };
  auto cta_of = [&](long long x) -> long long {
    if (!balanced) return x / per;
    int a = 0, b = p.num_ctas;   // bounds[a] <= x < bounds[b]
    while (b - a > 1) {
      const int m = (a + b) >> 1;
      if (bounds[m] <= x) a = m; else b = m;
    }
    return a;
  };
  // pass 2: segments. Tile k of request b starts at cost x_b + s0 + u k (x_b: the request's cost offset) and belongs
  // to CTA floor(cost / per); consecutive tiles of one request on one CTA form a segment.
  long long seg_carry = 0;
  for (int b0 = 0; b0 < B; b0 += kSchedThreads) {
    const int b = b0 + threadIdx.x;
    long long tiles = 0, x = 0, nseg = 0, c0 = 0;
    if (b < B) {
      tiles = (static_cast<long long>(p.seq_lens[b]) + tile - 1) / tile;
      x = p.seg_base[b];
      if (tiles > 0) {
        c0 = cta_of(x + s0);
        nseg = cta_of(x + s0 + u * (tiles - 1)) - c0 + 1;
      }
    }
    const long long base = seg_carry + block_exclusive_scan(nseg, warp_sums, &total_s);
    if (b < B) {
      p.seg_base[b] = static_cast<int32_t>(base);
      if (nseg > 0) {
        // CTAs after the previous request's last tile up to this one's first start at this request's first segment
        const long long prev = x > 0 ? cta_of(x - u) : -1;
        for (long long c = prev + 1; c <= c0 && c <= p.num_ctas; ++c) p.cta_seg[c] = static_cast<int32_t>(base);
      }
      for (long long j = 0; j < nseg; ++j) {
        const long long cta = c0 + j;
        long long k0 = cdiv(lo(cta) - x - s0, u), k1 = cdiv(lo(cta + 1) - x - s0, u);
        k0 = k0 > 0 ? k0 : 0;
        k1 = k1 < tiles ? k1 : tiles;
        const long long k = base + j;
        if (k < p.work_capacity) {
          p.work[4 * k + 0] = b;
          p.work[4 * k + 1] = static_cast<int32_t>(k0);
          p.work[4 * k + 2] = static_cast<int32_t>(k1);
          p.work[4 * k + 3] = 0;
        } else if (p.err) {
          atomicCAS(p.err, 0, kErrBadSegment);
        }
        if (j > 0 && cta <= p.num_ctas) p.cta_seg[cta] = static_cast<int32_t>(k);
      }
    }
    seg_carry += total_s;
    __syncthreads();
  }
  if (threadIdx.x == 0) p.seg_base[B] = static_cast<int32_t>(seg_carry);
  // CTAs after the last tile (and every CTA when there are no tiles) start at the end
  const long long last = total_cost > 0 ? cta_of(total_cost - u) : -1;
  for (long long c = last + 1 + threadIdx.x; c <= p.num_ctas; c += kSchedThreads)
    p.cta_seg[c] = static_cast<int32_t>(seg_carry);
}

cudaError_t launch_schedule(const ScheduleParams& p, cudaStream_t stream) {
  schedule_kernel<<<1, kSchedThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace belt
