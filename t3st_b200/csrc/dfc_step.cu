// Fused multi-tensor DFC-AdamW step for sm_100a.
//
// One launch updates every segment (parameter, or part of one) of the call.
// The segment list, the per-segment tile prefix and the hyper sets travel in
// the kernel's launch parameters (__grid_constant__, read through the
// constant cache), so a step needs no device-side descriptor table, no
// host->device copy and no allocation.  Each CTA owns one tile of kTile
// consecutive elements of one segment and finds its segment by binary search
// over the tile prefix.  A full, 16-byte-aligned tile is moved with 128-bit
// streaming loads/stores (ld.global.cs / st.global.cs: every byte is touched
// once per step), the loads of the four streams issued before any
// arithmetic.  The element arithmetic is ~80 instructions (two IEEE divides
// and an IEEE square root are needed for bit-exactness), so latency is hidden
// by occupancy rather than by unrolling: 256 threads x 1 float4 per stream,
// 32 registers, 8 CTAs (2048 threads) per SM, i.e. 128 KB of loads in flight
// per SM while other warps compute.  On the 62-tensor ResNet-18 step (11.2 M
// params, bench.py --steps 20 / 2000): this shape 232.8 / 234.2 G
// param-updates/s, 1.00 of the measured copy bandwidth; 2 float4 per stream
// per thread at 4 CTAs per SM 229.9-231.8; unroll 4 at 2 CTAs per SM 86% of
// the copy bandwidth.  Launched with programmatic dependent launch, so that
// back-to-back steps overlap one grid's last wave with the next grid's start
// (49.6 -> 47.8 us per step).
//
// The element arithmetic (remote/torch_fiber.py:90-116, explicit rounding)
// lives in dfc_step_elem.cuh, shared with the fused ZeRO-1 kernel.

#include <algorithm>
#include <vector>

#include "dfc_common.cuh"
#include "dfc_step_elem.cuh"

namespace dfc {
namespace {

// Tile shape (compile-time; the defaults are the measured best on B200).
#ifndef DFC_STEP_THREADS
#define DFC_STEP_THREADS 256
#endif
#ifndef DFC_STEP_UNROLL
#define DFC_STEP_UNROLL 1
#endif
#ifndef DFC_STEP_MIN_BLOCKS
#define DFC_STEP_MIN_BLOCKS 8
#endif
// resident CTAs per SM asked of the FP32-word kernels (modes PLAIN and
// SIGNFIBER), whose arithmetic needs more registers than the packed one
#ifndef DFC_STEP_MIN_BLOCKS_FP32
#define DFC_STEP_MIN_BLOCKS_FP32 6
#endif
constexpr int kThreads = DFC_STEP_THREADS;
constexpr int kVec = 4;
constexpr int kUnroll = DFC_STEP_UNROLL;
constexpr int kTile = kThreads * kVec * kUnroll;  // elements per CTA, FP32 parameters
// 16-bit parameters move fewer bytes per element (22 instead of 28), so a
// thread takes two quads per stream to keep as many bytes in flight: 2 quads
// at 5 CTAs per SM (48 registers, no spill) measured 275 G param-updates/s on
// the bf16 ResNet-18 step, 1 quad at 8 CTAs per SM 262, 2 quads at 4 CTAs 259
#ifndef DFC_STEP_UNROLL_16
#define DFC_STEP_UNROLL_16 2
#endif
#ifndef DFC_STEP_MIN_BLOCKS_16
#define DFC_STEP_MIN_BLOCKS_16 5
#endif
template <int PDT>
__host__ __device__ constexpr int unroll_of() { return PDT == DFC_DTYPE_F32 ? kUnroll : DFC_STEP_UNROLL_16; }
template <int PDT>
__host__ __device__ constexpr int tile_of() { return kThreads * kVec * unroll_of<PDT>(); }
int tile_elems(int32_t param_dtype) {
  return param_dtype == DFC_DTYPE_F32 ? kTile : kThreads * kVec * DFC_STEP_UNROLL_16;
}
// resident CTAs per SM asked of a kernel: packed FP32 parameters, FP32 words,
// or 16-bit parameters (default: as the moment format asks)
template <int MODE, int PDT>
__host__ __device__ constexpr int min_blocks_of() {
#ifdef DFC_STEP_MIN_BLOCKS_16
  if (PDT != DFC_DTYPE_F32) return DFC_STEP_MIN_BLOCKS_16;
#endif
  return MODE == DFC_MODE_PACKED ? DFC_STEP_MIN_BLOCKS : DFC_STEP_MIN_BLOCKS_FP32;
}

// SegArg.flags: bit 0 = the four-element vector path is aligned.
constexpr int32_t kFlagVec = 1;

struct SegArg {
  void* p;
  const void* g;
  uint32_t* m;
  uint32_t* v;
  int64_t n;
  int32_t hyper;
  int32_t flags;
};
static_assert(sizeof(SegArg) == 48, "SegArg layout");

template <int MAXS, int MAXH>
struct StepBatch {
  const float* dev_scale;
  int32_t n_segs;
  int32_t tile_base[MAXS + 1];  // tile_base[i] = first tile of segment i
  DfcHyper hyper[MAXH];
  SegArg seg[MAXS];
};

constexpr int kSmallSegs = 64, kSmallHypers = 8;
constexpr int kLargeSegs = 560, kLargeHypers = 32;
static_assert(sizeof(StepBatch<kLargeSegs, kLargeHypers>) <= 32000, "launch parameter limit");

// four consecutive elements of type DT at base[i] (i a multiple of 4)
template <int DT>
__device__ __forceinline__ float4 load4(const void* base, int64_t i) {
  if (DT == DFC_DTYPE_F32)
    return __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(base) + i));
  const uint2 b = __ldcs(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + i));
  return make_float4(from_bits16<DT>(b.x & 0xFFFFu), from_bits16<DT>(b.x >> 16),
                     from_bits16<DT>(b.y & 0xFFFFu), from_bits16<DT>(b.y >> 16));
}

template <int DT>
__device__ __forceinline__ void store4(void* base, int64_t i, const float4& v) {
  if (DT == DFC_DTYPE_F32) {
    __stcs(reinterpret_cast<float4*>(static_cast<float*>(base) + i), v);
  } else {
    const uint2 b = make_uint2(to_bits16<DT>(v.x) | (to_bits16<DT>(v.y) << 16),
                               to_bits16<DT>(v.z) | (to_bits16<DT>(v.w) << 16));
    __stcs(reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + i), b);
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* base, int64_t i) {
  if (DT == DFC_DTYPE_F32) return static_cast<const float*>(base)[i];
  return from_bits16<DT>(static_cast<const uint16_t*>(base)[i]);
}

template <int DT>
__device__ __forceinline__ void store1(void* base, int64_t i, float v) {
  if (DT == DFC_DTYPE_F32) static_cast<float*>(base)[i] = v;
  else static_cast<uint16_t*>(base)[i] = static_cast<uint16_t>(to_bits16<DT>(v));
}

template <int MODE, int PDT>
__device__ __forceinline__ void step4(const Scalars& s, float4& P, const float4& G, uint4& M,
                                      uint4& V) {
  step_elem<MODE, PDT>(s, P.x, G.x, M.x, V.x);
  step_elem<MODE, PDT>(s, P.y, G.y, M.y, V.y);
  step_elem<MODE, PDT>(s, P.z, G.z, M.z, V.z);
  step_elem<MODE, PDT>(s, P.w, G.w, M.w, V.w);
}

template <int MODE, int GDT, int PDT>
__device__ __forceinline__ void tile_full_vec(const SegArg& sg, int64_t base, const Scalars& s) {
  constexpr int U = unroll_of<PDT>();
  float4 P[U], G[U];
  uint4 M[U], V[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int64_t i = base + static_cast<int64_t>(u * kThreads + threadIdx.x) * kVec;
    P[u] = load4<PDT>(sg.p, i);
    G[u] = load4<GDT>(sg.g, i);
    M[u] = __ldcs(reinterpret_cast<const uint4*>(sg.m + i));
    V[u] = __ldcs(reinterpret_cast<const uint4*>(sg.v + i));
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int64_t i = base + static_cast<int64_t>(u * kThreads + threadIdx.x) * kVec;
    step4<MODE, PDT>(s, P[u], G[u], M[u], V[u]);
    store4<PDT>(sg.p, i, P[u]);
    __stcs(reinterpret_cast<uint4*>(sg.m + i), M[u]);
    __stcs(reinterpret_cast<uint4*>(sg.v + i), V[u]);
  }
}

template <int MODE, int GDT, int PDT>
__device__ __forceinline__ void tile_partial(const SegArg& sg, int64_t base, int64_t count,
                                             bool vec, const Scalars& s) {
  int64_t done = 0;
  if (vec) {
    const int64_t nv = count / kVec;
    for (int64_t j = threadIdx.x; j < nv; j += kThreads) {
      const int64_t i = base + j * kVec;
      float4 P = load4<PDT>(sg.p, i);
      const float4 G = load4<GDT>(sg.g, i);
      uint4 M = __ldcs(reinterpret_cast<const uint4*>(sg.m + i));
      uint4 V = __ldcs(reinterpret_cast<const uint4*>(sg.v + i));
      step4<MODE, PDT>(s, P, G, M, V);
      store4<PDT>(sg.p, i, P);
      __stcs(reinterpret_cast<uint4*>(sg.m + i), M);
      __stcs(reinterpret_cast<uint4*>(sg.v + i), V);
    }
    done = nv * kVec;
  }
  for (int64_t j = done + threadIdx.x; j < count; j += kThreads) {
    const int64_t i = base + j;
    float p = load1<PDT>(sg.p, i);
    uint32_t m = sg.m[i], v = sg.v[i];
    step_elem<MODE, PDT>(s, p, load1<GDT>(sg.g, i), m, v);
    store1<PDT>(sg.p, i, p);
    sg.m[i] = m;
    sg.v[i] = v;
  }
}

template <int MODE, int GDT, int PDT>
__device__ __forceinline__ void run_tile(const SegArg& sg, int64_t base, int64_t count,
                                         const Scalars& s) {
  const bool vec = (sg.flags & kFlagVec) != 0;
  if (vec && count == tile_of<PDT>()) tile_full_vec<MODE, GDT, PDT>(sg, base, s);
  else tile_partial<MODE, GDT, PDT>(sg, base, count, vec, s);
}

// One kernel per (moment format, gradient type, parameter type): a launch
// holds segments of a single type combination, so the hot FP32 kernel keeps
// its 32-register budget.
template <int MODE, int GDT, int PDT, int MAXS, int MAXH>
__global__ void __launch_bounds__(kThreads, (min_blocks_of<MODE, PDT>()))
    step_kernel(const __grid_constant__ StepBatch<MAXS, MAXH> b) {
  // Programmatic dependent launch: the next step's grid may start once every
  // CTA of this one has started, and waits (griddepcontrol.wait) for this
  // grid to finish before it touches memory.  Without a programmatic
  // predecessor the wait returns at once.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int32_t t = static_cast<int32_t>(blockIdx.x);
  int lo = 0, hi = b.n_segs;  // tile_base[lo] <= t < tile_base[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (b.tile_base[mid] <= t) lo = mid; else hi = mid;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // before the first global access
  const SegArg& sg = b.seg[lo];
  const Scalars s = load_scalars(b.hyper[sg.hyper], b.dev_scale);
  const int64_t base = static_cast<int64_t>(t - b.tile_base[lo]) * tile_of<PDT>();
  const int64_t count = min(static_cast<int64_t>(tile_of<PDT>()), sg.n - base);
  run_tile<MODE, GDT, PDT>(sg, base, count, s);
}

// type combination code: gradient type | parameter type << 2
int32_t types_of(const DfcSegment& s) { return s.grad_dtype | (s.param_dtype << 2); }

// Launch with programmatic stream serialization allowed: when the previous
// kernel on the stream is a step kernel (back-to-back optimizer steps), this
// grid's CTAs become resident during its tail instead of after it.
template <int MODE, int GDT, int PDT, int MAXS, int MAXH>
cudaError_t launch_one(const StepBatch<MAXS, MAXH>& b, int32_t grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel<MODE, GDT, PDT, MAXS, MAXH>, b);
}

template <int MODE, int MAXS, int MAXH>
cudaError_t launch_types(const StepBatch<MAXS, MAXH>& b, int32_t types, int32_t grid,
                         cudaStream_t st) {
  switch (types) {
    case 0: return launch_one<MODE, 0, 0>(b, grid, st);
    case 1: return launch_one<MODE, 1, 0>(b, grid, st);
    case 2: return launch_one<MODE, 2, 0>(b, grid, st);
    case 4: return launch_one<MODE, 0, 1>(b, grid, st);
    case 5: return launch_one<MODE, 1, 1>(b, grid, st);
    case 6: return launch_one<MODE, 2, 1>(b, grid, st);
    case 8: return launch_one<MODE, 0, 2>(b, grid, st);
    case 9: return launch_one<MODE, 1, 2>(b, grid, st);
    default: return launch_one<MODE, 2, 2>(b, grid, st);
  }
}

template <int MAXS, int MAXH>
int launch_batch(StepBatch<MAXS, MAXH>& b, int32_t mode, int32_t types, cudaStream_t st) {
  const int32_t tiles = b.tile_base[b.n_segs];
  if (tiles == 0) return DFC_OK;
  cudaError_t e;
  switch (mode) {
    case DFC_MODE_PLAIN: e = launch_types<DFC_MODE_PLAIN>(b, types, tiles, st); break;
    case DFC_MODE_SIGNFIBER: e = launch_types<DFC_MODE_SIGNFIBER>(b, types, tiles, st); break;
    default: e = launch_types<DFC_MODE_PACKED>(b, types, tiles, st); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_cuda_error(e);
    return DFC_ERR_CUDA;
  }
  return launch_status();
}

bool valid_dtype(int32_t t) { return t == DFC_DTYPE_F32 || t == DFC_DTYPE_BF16 || t == DFC_DTYPE_F16; }

uintptr_t elem_size(int32_t t) { return t == DFC_DTYPE_F32 ? 4 : 2; }

int validate(const DfcSegment& s, int32_t n_hypers) {
  if (s.numel < 0) return DFC_ERR_SIZE;
  if (s.numel == 0) return DFC_OK;
  if (!s.param || !s.grad || !s.exp_avg || !s.exp_avg_sq) return DFC_ERR_NULL;
  if (s.hyper < 0 || s.hyper >= n_hypers) return DFC_ERR_HYPER;
  if (!valid_dtype(s.grad_dtype) || !valid_dtype(s.param_dtype)) return DFC_ERR_DTYPE;
  if (!aligned(s.param, elem_size(s.param_dtype)) || !aligned(s.exp_avg, 4) ||
      !aligned(s.exp_avg_sq, 4) || !aligned(s.grad, elem_size(s.grad_dtype)))
    return DFC_ERR_ALIGN;
  if ((s.numel + kTile - 1) / kTile > INT32_MAX / 2) return DFC_ERR_SIZE;
  return DFC_OK;
}

SegArg to_arg(const DfcSegment& s, int32_t local_hyper) {
  SegArg a;
  a.p = s.param;
  a.g = s.grad;
  a.m = s.exp_avg;
  a.v = s.exp_avg_sq;
  a.n = s.numel;
  a.hyper = local_hyper;
  // a vector of four elements: 16 bytes of FP32, 8 bytes of a 16-bit type
  const bool vec = aligned(s.param, 4 * elem_size(s.param_dtype)) && aligned(s.exp_avg, 16) &&
                   aligned(s.exp_avg_sq, 16) && aligned(s.grad, 4 * elem_size(s.grad_dtype));
  a.flags = vec ? kFlagVec : 0;
  return a;
}

// Pack the segments of one type combination into as few launches as the
// per-launch capacity allows.  A batch closes when it holds MAXS segments,
// MAXH distinct hyper sets, or would pass INT32_MAX tiles.
template <int MAXS, int MAXH>
int run_batches(const DfcSegment* segs, int32_t n, const DfcHyper* hypers, int32_t n_hypers,
                int32_t mode, int32_t types, const float* dscale, cudaStream_t st) {
  StepBatch<MAXS, MAXH> b;
  std::vector<int32_t> local(static_cast<size_t>(n_hypers), -1);
  std::vector<int32_t> used;
  auto reset = [&]() {
    for (int32_t g : used) local[g] = -1;
    used.clear();
    b.dev_scale = dscale;
    b.n_segs = 0;
    b.tile_base[0] = 0;
  };
  reset();
  for (int32_t i = 0; i < n; ++i) {
    const DfcSegment& s = segs[i];
    if (s.numel == 0 || types_of(s) != types) continue;
    const int64_t tile = tile_elems(s.param_dtype);
    const int32_t tiles = static_cast<int32_t>((s.numel + tile - 1) / tile);
    const bool need_hyper = local[s.hyper] < 0;
    if (b.n_segs == MAXS || (need_hyper && static_cast<int>(used.size()) == MAXH) ||
        b.tile_base[b.n_segs] > INT32_MAX - tiles) {
      int rc = launch_batch(b, mode, types, st);
      if (rc != DFC_OK) return rc;
      reset();
    }
    if (local[s.hyper] < 0) {
      local[s.hyper] = static_cast<int32_t>(used.size());
      b.hyper[used.size()] = hypers[s.hyper];
      used.push_back(s.hyper);
    }
    b.seg[b.n_segs] = to_arg(s, local[s.hyper]);
    b.tile_base[b.n_segs + 1] = b.tile_base[b.n_segs] + tiles;
    ++b.n_segs;
  }
  return b.n_segs ? launch_batch(b, mode, types, st) : DFC_OK;
}

template <int MAXS, int MAXH>
int run_all(const DfcSegment* segs, int32_t n, const DfcHyper* hypers, int32_t n_hypers,
            int32_t mode, const float* dscale, cudaStream_t st) {
  bool present[16] = {};
  for (int32_t i = 0; i < n; ++i)
    if (segs[i].numel > 0) present[types_of(segs[i])] = true;
  for (int32_t types = 0; types < 16; ++types) {
    if (!present[types]) continue;
    const int rc = run_batches<MAXS, MAXH>(segs, n, hypers, n_hypers, mode, types, dscale, st);
    if (rc != DFC_OK) return rc;
  }
  return DFC_OK;
}

// ---- moment-format conversion -------------------------------------------
// PACK: FP32 word -> packed word; otherwise packed -> FP32.  Bit 31 passes
// through (sign of a first moment, payload of a second moment), except that
// a first-moment NaN packs to the canonical +NaN word.
template <bool PACK, bool SECOND>
__global__ void convert_kernel(uint32_t* w, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint32_t x = w[i];
    const uint32_t sign = x & 0x80000000u;
    if (PACK) w[i] = SECOND ? sign | enc_mag(x & 0x7FFFFFFFu) : enc_signed_bits(x);
    else w[i] = sign | dec_mag(x & 0x7FFFFFFFu);
  }
}

int convert(uint32_t* w, int64_t n, bool pack, bool second, void* stream) {
  if (n < 0) return DFC_ERR_SIZE;
  if (n == 0) return DFC_OK;
  if (!w) return DFC_ERR_NULL;
  if (!aligned(w, 4)) return DFC_ERR_ALIGN;
  const int64_t want = (n + 255) / 256;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto grid = [&](auto kernel) {
    return static_cast<int>(std::min<int64_t>(want, resident_ctas(kernel, 256)));
  };
  if (pack && second) convert_kernel<true, true><<<grid(convert_kernel<true, true>), 256, 0, st>>>(w, n);
  else if (pack) convert_kernel<true, false><<<grid(convert_kernel<true, false>), 256, 0, st>>>(w, n);
  else convert_kernel<false, false><<<grid(convert_kernel<false, false>), 256, 0, st>>>(w, n);
  return launch_status();
}

}  // namespace
}  // namespace dfc

extern "C" int dfc_mt_step(const DfcSegment* segments, int32_t n_segments, const DfcHyper* hypers,
                           int32_t n_hypers, int32_t mode, const float* device_grad_scale,
                           void* stream) {
  using namespace dfc;
  if (n_segments < 0 || n_hypers < 0) return DFC_ERR_SIZE;
  if (mode != DFC_MODE_PLAIN && mode != DFC_MODE_SIGNFIBER && mode != DFC_MODE_PACKED)
    return DFC_ERR_MODE;
  if (n_segments == 0) return DFC_OK;
  if (!segments || (!hypers && n_hypers > 0)) return DFC_ERR_NULL;
  for (int32_t i = 0; i < n_segments; ++i) {
    const int rc = validate(segments[i], n_hypers);
    if (rc != DFC_OK) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_segments <= kSmallSegs && n_hypers <= kSmallHypers)
    return run_all<kSmallSegs, kSmallHypers>(segments, n_segments, hypers, n_hypers, mode,
                                             device_grad_scale, st);
  return run_all<kLargeSegs, kLargeHypers>(segments, n_segments, hypers, n_hypers, mode,
                                           device_grad_scale, st);
}

extern "C" int dfc_pack_moments(uint32_t* words, int64_t n, int32_t second, void* stream) {
  return dfc::convert(words, n, true, second != 0, stream);
}

extern "C" int dfc_unpack_moments(uint32_t* words, int64_t n, int32_t second, void* stream) {
  return dfc::convert(words, n, false, second != 0, stream);
}
