// Per-buffer gradient statistics (sum of squares, max |g|, non-finite count)
// and the global-norm clip coefficient.
//
// Pass 1: tiles of kTile elements of one buffer; a persistent grid (the CTAs
// resident at once) walks them, each CTA prefetching its next tile while it
// reduces the current one.  Per tile, each thread accumulates its elements
// (sum of squares in double), the CTA reduces with warp shuffles
// (__shfl_xor_sync butterfly) and one shared-memory step across warps, and
// writes one partial record per tile to scratch.
// Pass 2: one CTA per buffer folds that buffer's partial records in a fixed
// order.  No atomics anywhere, so the result depends only on the input and
// the tile size, never on scheduling.
#include <algorithm>
#include <math.h>

#include "dfc_common.cuh"
#include "dfc_step_elem.cuh"

namespace dfc {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 8192;
constexpr int kMaxBufs = 1000;

struct BufArg {
  const void* g;
  int64_t n;
  int32_t dtype;  // DFC_DTYPE_*
  int32_t vec;    // FP32 and 16-byte aligned
};

struct StatsBatch {
  DfcGradStats* partial;  // scratch, one record per tile of this batch
  DfcGradStats* out;      // one record per buffer of this batch
  int32_t n_bufs;
  int32_t tile_base[kMaxBufs + 1];
  BufArg buf[kMaxBufs];
};
static_assert(sizeof(StatsBatch) <= 32000, "launch parameter limit");

struct Acc {
  double s;
  float a;
  long long bad;
};

__device__ __forceinline__ void acc_add(Acc& acc, float x) {
  acc.s += static_cast<double>(x) * static_cast<double>(x);
  acc.a = fmaxf(acc.a, fabsf(x));
  acc.bad += isfinite(x) ? 0 : 1;
}

__device__ __forceinline__ void acc_merge(Acc& acc, const Acc& o) {
  acc.s += o.s;
  acc.a = fmaxf(acc.a, o.a);
  acc.bad += o.bad;
}

__device__ __forceinline__ Acc warp_fold(Acc acc) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Acc o;
    o.s = __shfl_xor_sync(0xFFFFFFFFu, acc.s, off);
    o.a = __shfl_xor_sync(0xFFFFFFFFu, acc.a, off);
    o.bad = __shfl_xor_sync(0xFFFFFFFFu, acc.bad, off);
    acc_merge(acc, o);
  }
  return acc;
}

__device__ __forceinline__ float load1(const BufArg& b, int64_t i) {
  if (b.dtype == DFC_DTYPE_BF16) return from_bits16<DFC_DTYPE_BF16>(static_cast<const uint16_t*>(b.g)[i]);
  if (b.dtype == DFC_DTYPE_F16) return from_bits16<DFC_DTYPE_F16>(static_cast<const uint16_t*>(b.g)[i]);
  return static_cast<const float*>(b.g)[i];
}

constexpr int kLoads = kTile / 4 / kThreads;  // float4 loads per thread in a full tile

// Tile t's buffer (binary search over the tile prefix) and element range.
struct TileRef {
  const BufArg* buf;
  int64_t base;
  int64_t count;
};

__device__ __forceinline__ TileRef tile_ref(const StatsBatch& b, int32_t t) {
  int lo = 0, hi = b.n_bufs;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (b.tile_base[mid] <= t) lo = mid; else hi = mid;
  }
  TileRef r;
  r.buf = &b.buf[lo];
  r.base = static_cast<int64_t>(t - b.tile_base[lo]) * kTile;
  r.count = min(static_cast<int64_t>(kTile), b.buf[lo].n - r.base);
  return r;
}

__device__ __forceinline__ bool full_vec(const TileRef& r) { return r.buf->vec && r.count == kTile; }

__device__ __forceinline__ void load_tile(const TileRef& r, float4 (&x)[kLoads]) {
  const float4* g4 = reinterpret_cast<const float4*>(static_cast<const float*>(r.buf->g) + r.base);
#pragma unroll
  for (int u = 0; u < kLoads; ++u) x[u] = __ldcs(g4 + threadIdx.x + u * kThreads);
}

// This thread's share of one tile, in the order j = threadIdx.x, +kThreads, ...
// (a full FP32 tile arrives preloaded in x).
__device__ __forceinline__ Acc tile_acc(const TileRef& r, const float4 (&x)[kLoads], bool pre) {
  Acc acc{0.0, 0.0f, 0};
  if (pre) {
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      acc_add(acc, x[u].x);
      acc_add(acc, x[u].y);
      acc_add(acc, x[u].z);
      acc_add(acc, x[u].w);
    }
    return acc;
  }
  const BufArg& buf = *r.buf;
  int64_t done = 0;
  if (buf.vec) {
    const float4* g4 = reinterpret_cast<const float4*>(static_cast<const float*>(buf.g) + r.base);
    const int64_t nv = r.count / 4;
    for (int64_t j = threadIdx.x; j < nv; j += kThreads) {
      const float4 v = __ldcs(g4 + j);
      acc_add(acc, v.x);
      acc_add(acc, v.y);
      acc_add(acc, v.z);
      acc_add(acc, v.w);
    }
    done = nv * 4;
  }
  for (int64_t j = done + threadIdx.x; j < r.count; j += kThreads) acc_add(acc, load1(buf, r.base + j));
  return acc;
}

// Persistent: CTA c takes tiles c, c + gridDim.x, ...  A full FP32 tile's
// loads are issued before the previous tile is reduced, so the SM keeps
// loads in flight through the block reduction.  Each tile's record is the
// same as with one CTA per tile: the per-thread order, the warp butterfly
// and the fixed fold over warps do not depend on the grid.
__global__ void __launch_bounds__(kThreads, 3) stats_partial_kernel(const __grid_constant__ StatsBatch b) {
  __shared__ Acc part[2][kWarps];  // double-buffered: one barrier per tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t tiles = b.tile_base[b.n_bufs];
  int32_t t = static_cast<int32_t>(blockIdx.x);
  if (t >= tiles) return;
  TileRef cur = tile_ref(b, t);
  float4 x[kLoads];
  bool pre = full_vec(cur);
  if (pre) load_tile(cur, x);
  for (int it = 0; t < tiles; t += static_cast<int32_t>(gridDim.x), ++it) {
    Acc acc = tile_acc(cur, x, pre);
    const int32_t tn = t + static_cast<int32_t>(gridDim.x);
    TileRef nxt = cur;
    bool pre_n = false;
    if (tn < tiles) {
      nxt = tile_ref(b, tn);
      pre_n = full_vec(nxt);
      if (pre_n) load_tile(nxt, x);  // x is free: this tile's values are in acc
    }
    acc = warp_fold(acc);
    if (lane == 0) part[it & 1][warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      Acc tot = part[it & 1][0];
      for (int w = 1; w < kWarps; ++w) acc_merge(tot, part[it & 1][w]);
      DfcGradStats rec;
      rec.sumsq = tot.s;
      rec.amax = tot.a;
      rec.reserved = 0;
      rec.nonfinite = tot.bad;
      b.partial[t] = rec;
    }
    cur = nxt;
    pre = pre_n;
  }
}

// One CTA per buffer folds that buffer's partial records: thread i takes
// records i, i + kThreads, ... in order (loads batched kBatch at a time), then
// the warp butterfly and a fixed fold over warps.  Deterministic.
constexpr int kBatch = 4;

__global__ void __launch_bounds__(kThreads) stats_final_kernel(const __grid_constant__ StatsBatch b) {
  const int buf = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t t0 = b.tile_base[buf], t1 = b.tile_base[buf + 1];
  Acc acc{0.0, 0.0f, 0};
  for (int32_t t = t0 + threadIdx.x; t < t1; t += kBatch * kThreads) {
    DfcGradStats r[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (t + u * kThreads < t1) r[u] = b.partial[t + u * kThreads];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (t + u * kThreads < t1) {
        Acc o{r[u].sumsq, r[u].amax, r[u].nonfinite};
        acc_merge(acc, o);
      }
    }
  }
  acc = warp_fold(acc);
  __shared__ Acc part[kWarps];
  if (lane == 0) part[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    Acc tot = part[0];
    for (int w = 1; w < kWarps; ++w) acc_merge(tot, part[w]);
    DfcGradStats r;
    r.sumsq = tot.s;
    r.amax = tot.a;
    r.reserved = 0;
    r.nonfinite = tot.bad;
    b.out[buf] = r;
  }
}

int64_t tiles_of(int64_t n) { return (n + kTile - 1) / kTile; }

int validate(const DfcGradRef& r) {
  if (r.numel < 0) return DFC_ERR_SIZE;
  if (r.grad_dtype != DFC_DTYPE_F32 && r.grad_dtype != DFC_DTYPE_BF16 &&
      r.grad_dtype != DFC_DTYPE_F16)
    return DFC_ERR_DTYPE;
  if (r.numel == 0) return DFC_OK;
  if (!r.grad) return DFC_ERR_NULL;
  if (!aligned(r.grad, r.grad_dtype == DFC_DTYPE_F32 ? 4 : 2)) return DFC_ERR_ALIGN;
  if (tiles_of(r.numel) > INT32_MAX / 2) return DFC_ERR_SIZE;
  return DFC_OK;
}

}  // namespace

// Shared with the scratch-free variant: launches both passes over `grads`,
// with partial records at `partial` (n_tiles_total records).
int grad_stats_launch(const DfcGradRef* grads, int32_t n_grads, DfcGradStats* out,
                      DfcGradStats* partial, cudaStream_t st) {
  StatsBatch b;
  int64_t tile_off = 0;
  int32_t first = 0;
  while (first < n_grads) {
    b.partial = partial + tile_off;
    b.out = out + first;
    b.n_bufs = 0;
    b.tile_base[0] = 0;
    int32_t i = first;
    // Every buffer gets a record, so empty buffers take one (empty) tile.
    while (i < n_grads && b.n_bufs < kMaxBufs) {
      const int64_t tl = std::max<int64_t>(1, tiles_of(grads[i].numel));
      if (b.tile_base[b.n_bufs] + tl > INT32_MAX / 2 && b.n_bufs > 0) break;
      BufArg a;
      a.g = grads[i].grad;
      a.n = grads[i].numel;
      a.dtype = grads[i].grad_dtype;
      a.vec = grads[i].grad_dtype == DFC_DTYPE_F32 && aligned(grads[i].grad, 16);
      b.buf[b.n_bufs] = a;
      b.tile_base[b.n_bufs + 1] = b.tile_base[b.n_bufs] + static_cast<int32_t>(tl);
      ++b.n_bufs;
      ++i;
    }
    const int32_t tiles = b.tile_base[b.n_bufs];
    const int32_t grid = static_cast<int32_t>(std::min<int64_t>(tiles, static_cast<int64_t>(sm_count()) * 3));
    stats_partial_kernel<<<grid, kThreads, 0, st>>>(b);
    stats_final_kernel<<<b.n_bufs, kThreads, 0, st>>>(b);
    const int rc = launch_status();
    if (rc != DFC_OK) return rc;
    tile_off += tiles;
    first = i;
  }
  return DFC_OK;
}

size_t grad_stats_records(const DfcGradRef* grads, int32_t n_grads) {
  size_t total = 0;
  for (int32_t i = 0; i < n_grads; ++i)
    total += static_cast<size_t>(std::max<int64_t>(1, tiles_of(std::max<int64_t>(0, grads[i].numel))));
  return total;
}

int grad_stats_validate(const DfcGradRef* grads, int32_t n_grads) {
  if (n_grads < 0) return DFC_ERR_SIZE;
  if (n_grads > 0 && !grads) return DFC_ERR_NULL;
  for (int32_t i = 0; i < n_grads; ++i) {
    const int rc = validate(grads[i]);
    if (rc != DFC_OK) return rc;
  }
  return DFC_OK;
}

namespace {

__global__ void __launch_bounds__(kThreads)
    clip_kernel(const DfcGradStats* stats, int32_t n, float max_norm, float* coef, float* norm) {
  double s = 0.0;
  for (int32_t i = threadIdx.x; i < n; i += kThreads) s += stats[i].sumsq;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
  __shared__ double part[kWarps];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = part[0];
    for (int w = 1; w < kWarps; ++w) tot += part[w];
    const float total = static_cast<float>(sqrt(tot));
    const float c = fminf(__fdiv_rn(max_norm, __fadd_rn(total, 1e-6f)), 1.0f);
    if (coef) *coef = c;
    if (norm) *norm = total;
  }
}

}  // namespace
}  // namespace dfc

extern "C" size_t dfc_grad_stats_scratch_bytes(const DfcGradRef* grads, int32_t n_grads) {
  if (n_grads <= 0 || !grads) return 0;
  return dfc::grad_stats_records(grads, n_grads) * sizeof(DfcGradStats);
}

extern "C" int dfc_grad_stats(const DfcGradRef* grads, int32_t n_grads, DfcGradStats* out,
                              void* scratch, size_t scratch_bytes, void* stream) {
  using namespace dfc;
  int rc = grad_stats_validate(grads, n_grads);
  if (rc != DFC_OK) return rc;
  if (n_grads == 0) return DFC_OK;
  if (!out || !scratch) return DFC_ERR_NULL;
  if (!aligned(out, 8) || !aligned(scratch, 8)) return DFC_ERR_ALIGN;
  if (scratch_bytes < grad_stats_records(grads, n_grads) * sizeof(DfcGradStats))
    return DFC_ERR_SCRATCH;
  return grad_stats_launch(grads, n_grads, out, static_cast<DfcGradStats*>(scratch),
                           static_cast<cudaStream_t>(stream));
}

extern "C" int dfc_clip_coef(const DfcGradStats* stats, int32_t n_stats, float max_norm,
                             float* out_coef, float* out_norm, void* stream) {
  using namespace dfc;
  if (n_stats < 0) return DFC_ERR_SIZE;
  if (!stats && n_stats > 0) return DFC_ERR_NULL;
  if (!out_coef && !out_norm) return DFC_OK;
  if (!aligned(stats, 8) || !aligned(out_coef, 4) || !aligned(out_norm, 4)) return DFC_ERR_ALIGN;
  clip_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(stats, n_stats, max_norm,
                                                                      out_coef, out_norm);
  return launch_status();
}
