// ZeRO-1 shard step fused with its collectives over NVLink peer memory.
//
// With the FP32 parameter vector and the bf16 compressed gradients in
// symmetric (peer-mapped) memory on every rank, one kernel does what NCCL
// reduce-scatter + dfc_mt_step + NCCL all-gather do, for this rank's pieces:
//
//   g      = (sum over ranks q = 0..N-1, in that order, of comp_q[j]) in FP32
//   p, m, v = DFC-AdamW step (same element arithmetic as dfc_mt_step)
//   param_q[j] = p  for every rank q (plain 128-bit stores to peer memory)
//
// Gradients cross NVLink once (2 B per element per peer) and parameters
// once (4 B per element per peer), the reduction happens in registers in
// FP32 (deterministic order, no bf16 re-rounding of partial sums), and no
// reduce-scatter output buffer or all-gather staging is written to HBM.  Only
// plain loads and stores touch peer memory (no TMA).
//
// NVLS form (multicast addresses given): the NVSwitch does the reduction
// (multimem.ld_reduce, FP32 accumulation, bf16 result) and replicates the
// parameter stores (multimem.st), so each value crosses this GPU's links
// once instead of once per peer.  dfc_multicast_sum_bf16 reads the switch's
// sums back, for checking.
//
// dfc_zero_fused_step_ef adds the next bucket's gradient compression to the
// same grid: its tiles are spread evenly among the step's, so the step's
// NVLink traffic and the compression's HBM traffic run side by side in one
// kernel instead of two kernels on two streams competing for SMs.
//
// dfc_peer_barrier orders the ranks around it: each rank writes an epoch to
// its slot in every peer's signal array (release, system scope) and then
// waits for every peer's slot in its own array (acquire, system scope), for at
// most a time limit; a rank that gives up sets an error flag and returns.
#include <algorithm>
#include <vector>

#include "dfc_common.cuh"
#include "dfc_compress_elem.cuh"
#include "dfc_step_elem.cuh"

namespace dfc {
namespace {

constexpr int kThreads = 256;
constexpr int kVec = 8;                      // elements per thread per tile (two quads)
constexpr int kTile = kThreads * kVec;       // 2048 elements per CTA
constexpr int kMaxPeers = DFC_MAX_PEERS;

struct PeerSegArg {
  int64_t offset;  // flat element index of the segment's first element
  int64_t n;
  uint32_t* m;
  uint32_t* v;
  int32_t hyper;
  int32_t vec;     // offset and moment words allow the quad path
};

template <int MAXS, int MAXH>
struct ZeroBatch {
  const uint16_t* comp[kMaxPeers];  // every rank's compressed gradients (bf16 bits)
  float* param[kMaxPeers];          // every rank's flat FP32 parameters
  const uint16_t* comp_mc;          // multicast address of the gradients (nvls kernel)
  float* param_mc;                  // multicast address of the parameters (nvls kernel)
  const float* dev_scale;
  const int32_t* error;             // a barrier's give-up flag, or null
  const float* cgrad;               // compression run in the same grid (dfc_zero_fused_step_ef)
  uint16_t* ccomp;
  uint16_t* cresid;
  int64_t cquads;                   // its length in quads
  int32_t ctiles;                   // its tiles of kTile elements (0: none)
  int32_t n_peers;
  int32_t rank;
  int32_t n_segs;
  int32_t tile_base[MAXS + 1];
  DfcHyper hyper[MAXH];
  PeerSegArg seg[MAXS];
};

constexpr int kMaxSegs = 512, kMaxHypers = 16;
static_assert(sizeof(ZeroBatch<kMaxSegs, kMaxHypers>) <= 32000, "launch parameter limit");

// The switch's sum of element j over every rank: the aligned bf16x2 word
// that holds j is reduced (FP32 accumulation, bf16 result) and j's half kept.
// The word never leaves the 4-byte granule of a valid element.
__device__ __forceinline__ float nvls_sum1(const uint16_t* mc, int64_t j) {
  uint32_t w;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.bf16x2 %0, [%1];"
               : "=r"(w)
               : "l"(mc + (j & ~int64_t(1)))
               : "memory");
  return u2f((j & 1) ? (w & 0xFFFF0000u) : (w << 16));
}

__device__ __forceinline__ void nvls_sum8(const uint16_t* mc, float (&g)[8]) {
  uint32_t r[4];
  asm volatile(
      "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "l"(mc)
      : "memory");
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    g[2 * k] = u2f(r[k] << 16);
    g[2 * k + 1] = u2f(r[k] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ void nvls_sum4(const uint16_t* mc, float (&g)[4]) {
  uint32_t r[2];
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v2.bf16x2 {%0, %1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "l"(mc)
               : "memory");
  g[0] = u2f(r[0] << 16);
  g[1] = u2f(r[0] & 0xFFFF0000u);
  g[2] = u2f(r[1] << 16);
  g[3] = u2f(r[1] & 0xFFFF0000u);
}

// Q quads (4 consecutive elements each) of one segment per thread, at local
// offsets l[0..Q).  Thread t of a CTA takes quads t and t + 256 of its tile,
// so every warp-wide access -- above all the parameter stores that cross
// NVLink -- covers 32 consecutive quads: whole 32-byte sectors, no
// half-filled remote writes.  All remote loads of the Q quads are issued
// before the first use so their latencies overlap.
//
// Plain form (NVLS false): g = comp_0[j] + comp_1[j] + ... in FP32, rank
// order, over NP ranks (NP = 2, 4, 8 at compile time; 0 = any, predicated),
// and the new parameters are stored to every rank's copy.  NVLS form: the
// switch's sum (multimem.ld_reduce) and one multicast store (multimem.st).
template <int MODE, int NP, bool NVLS, int Q, int MAXS, int MAXH>
__device__ __forceinline__ void quads(const ZeroBatch<MAXS, MAXH>& b, const PeerSegArg& sg,
                                      const int64_t (&l)[Q], const Scalars& s) {
  constexpr int kLoads = NVLS ? 1 : (NP ? NP : kMaxPeers);
  const int np = NP ? NP : b.n_peers;
  float g[Q][4];
  uint2 c[Q][kLoads];
#pragma unroll
  for (int u = 0; u < Q; ++u) {
    const int64_t j = sg.offset + l[u];
    if (NVLS) {
      nvls_sum4(b.comp_mc + j, g[u]);
    } else {
#pragma unroll
      for (int q = 0; q < kLoads; ++q)
        if (NP || q < np) c[u][q] = __ldcs(reinterpret_cast<const uint2*>(b.comp[q] + j));
    }
  }
  float4 p[Q];
  uint4 m[Q], v[Q];
#pragma unroll
  for (int u = 0; u < Q; ++u) {
    p[u] = __ldcs(reinterpret_cast<const float4*>(b.param[b.rank] + sg.offset + l[u]));
    m[u] = __ldcs(reinterpret_cast<const uint4*>(sg.m + l[u]));
    v[u] = __ldcs(reinterpret_cast<const uint4*>(sg.v + l[u]));
  }
#pragma unroll
  for (int u = 0; u < Q; ++u) {
    if (!NVLS) {
      g[u][0] = u2f(c[u][0].x << 16);
      g[u][1] = u2f(c[u][0].x & 0xFFFF0000u);
      g[u][2] = u2f(c[u][0].y << 16);
      g[u][3] = u2f(c[u][0].y & 0xFFFF0000u);
#pragma unroll
      for (int q = 1; q < kLoads; ++q) {
        if (NP || q < np) {
          g[u][0] = __fadd_rn(g[u][0], u2f(c[u][q].x << 16));
          g[u][1] = __fadd_rn(g[u][1], u2f(c[u][q].x & 0xFFFF0000u));
          g[u][2] = __fadd_rn(g[u][2], u2f(c[u][q].y << 16));
          g[u][3] = __fadd_rn(g[u][3], u2f(c[u][q].y & 0xFFFF0000u));
        }
      }
    }
    step_elem<MODE>(s, p[u].x, g[u][0], m[u].x, v[u].x);
    step_elem<MODE>(s, p[u].y, g[u][1], m[u].y, v[u].y);
    step_elem<MODE>(s, p[u].z, g[u][2], m[u].z, v[u].z);
    step_elem<MODE>(s, p[u].w, g[u][3], m[u].w, v[u].w);
    __stcs(reinterpret_cast<uint4*>(sg.m + l[u]), m[u]);
    __stcs(reinterpret_cast<uint4*>(sg.v + l[u]), v[u]);
    const int64_t j = sg.offset + l[u];
    if (NVLS) {
      asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(b.param_mc + j),
                   "f"(p[u].x), "f"(p[u].y), "f"(p[u].z), "f"(p[u].w)
                   : "memory");
    } else {
#pragma unroll
      for (int q = 0; q < (NP ? NP : kMaxPeers); ++q)
        if (NP || q < np) __stcs(reinterpret_cast<float4*>(b.param[q] + j), p[u]);
    }
  }
}

// One element.  Plain form: peer loads, FP32 sum in rank order, peer stores.
// NVLS form: the switch's sum and one multicast store, as in quads, so
// every element of a bucket follows the switch's rounding.
template <int MODE, bool NVLS, int MAXS, int MAXH>
__device__ __forceinline__ void scalar1(const ZeroBatch<MAXS, MAXH>& b, const PeerSegArg& sg,
                                        int64_t local, const Scalars& s) {
  const int64_t j = sg.offset + local;
  float g;
  if (NVLS) {
    g = nvls_sum1(b.comp_mc, j);
  } else {
    g = bf16_bits_to_f32(b.comp[0][j]);
    for (int q = 1; q < b.n_peers; ++q) g = __fadd_rn(g, bf16_bits_to_f32(b.comp[q][j]));
  }
  float p = b.param[b.rank][j];
  uint32_t m = sg.m[local], v = sg.v[local];
  step_elem<MODE>(s, p, g, m, v);
  sg.m[local] = m;
  sg.v[local] = v;
  if (NVLS) {
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(b.param_mc + j), "f"(p)
                 : "memory");
  } else {
    for (int q = 0; q < b.n_peers; ++q) b.param[q][j] = p;
  }
}

// CTA c handles tiles c, c + gridDim.x, ...: one tile per CTA when the grid
// has a CTA per tile, a persistent walk when the grid is capped so that a
// kernel on another stream (the next bucket's compression) keeps SMs.
//
// With a compression in the grid the tiles are T = F step tiles + C
// compression tiles, and tile t is a step tile exactly when
// floor((t+1) F / T) > floor(t F / T): step tile floor(t F / T), else
// compression tile t - floor(t F / T).  Both kinds are spread evenly over the
// grid, in address order within each kind.
template <int MODE, int NP, bool NVLS, int MAXS, int MAXH>
__global__ void __launch_bounds__(kThreads, 4)
    zero_step_kernel(const __grid_constant__ ZeroBatch<MAXS, MAXH> b) {
  const int64_t ftiles = b.tile_base[b.n_segs];
  const int64_t total = ftiles + b.ctiles;
  bool ready = false, failed = false;
  for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
    int64_t ft = u;
    if (b.ctiles) {
      ft = u * ftiles / total;
      if ((u + 1) * ftiles / total == ft) {
        compress_tile<kThreads>(b.cgrad, b.ccomp, b.cresid, b.cquads, u - ft);
        continue;
      }
    }
    if (!ready) {
      // Launched as a programmatic dependent of the barrier (compression
      // tiles then start while it waits): the step waits here for the
      // barrier grid to finish.  Otherwise this returns at once.
      asm volatile("griddepcontrol.wait;" ::: "memory");
      // A barrier before this kernel gave up: a peer may be stalled or gone,
      // so neither its gradients nor its parameter copy may be touched.  The
      // compression touches this rank's memory only and runs regardless.
      failed = b.error && *static_cast<const volatile int32_t*>(b.error) != 0;
      ready = true;
    }
    if (failed) {
      if (b.ctiles == 0) return;
      continue;
    }
    const int32_t t = static_cast<int32_t>(ft);
    int lo = 0, hi = b.n_segs;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (b.tile_base[mid] <= t) lo = mid; else hi = mid;
    }
    const PeerSegArg& sg = b.seg[lo];
    const Scalars s = load_scalars(b.hyper[sg.hyper], b.dev_scale);
    const int64_t base = static_cast<int64_t>(t - b.tile_base[lo]) * kTile;
    const int64_t count = min(static_cast<int64_t>(kTile), sg.n - base);
    const int64_t nq = sg.vec ? count / 4 : 0;  // whole quads of this tile
    const int64_t k0 = threadIdx.x, k1 = threadIdx.x + kThreads;
    if (k1 < nq) {
      const int64_t l[2] = {base + 4 * k0, base + 4 * k1};
      quads<MODE, NP, NVLS, 2>(b, sg, l, s);
    } else if (k0 < nq) {
      const int64_t l[1] = {base + 4 * k0};
      quads<MODE, NP, NVLS, 1>(b, sg, l, s);
    }
    for (int64_t k = nq * 4 + threadIdx.x; k < count; k += kThreads)
      scalar1<MODE, NVLS>(b, sg, base + k, s);
  }
}

// pdl: launched with programmatic stream serialization, so the grid may
// start while the previous kernel on the stream runs, once that kernel allows
// it (dfc_peer_barrier does, as it starts).
template <typename Batch>
cudaError_t launch_kernel(void (*kernel)(Batch), const Batch& b, int32_t grid, bool pdl,
                          cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, b);
}

template <int MODE, int MAXS, int MAXH>
cudaError_t launch_np(const ZeroBatch<MAXS, MAXH>& b, int32_t grid, bool pdl, cudaStream_t st) {
  if (b.comp_mc) return launch_kernel(zero_step_kernel<MODE, 0, true, MAXS, MAXH>, b, grid, pdl, st);
  switch (b.n_peers) {
    case 2: return launch_kernel(zero_step_kernel<MODE, 2, false, MAXS, MAXH>, b, grid, pdl, st);
    case 4: return launch_kernel(zero_step_kernel<MODE, 4, false, MAXS, MAXH>, b, grid, pdl, st);
    case 8: return launch_kernel(zero_step_kernel<MODE, 8, false, MAXS, MAXH>, b, grid, pdl, st);
    default: return launch_kernel(zero_step_kernel<MODE, 0, false, MAXS, MAXH>, b, grid, pdl, st);
  }
}

// One CTA per tile (ctas_per_sm <= 0), or at most ctas_per_sm CTAs per SM.
template <int MAXS, int MAXH>
int launch(const ZeroBatch<MAXS, MAXH>& b, int32_t mode, int32_t ctas_per_sm, bool pdl,
           cudaStream_t st) {
  const int64_t tiles = static_cast<int64_t>(b.tile_base[b.n_segs]) + b.ctiles;
  if (tiles == 0) return DFC_OK;
  if (tiles > INT32_MAX) return DFC_ERR_SIZE;
  int32_t grid = static_cast<int32_t>(tiles);
  if (ctas_per_sm > 0) grid = static_cast<int32_t>(std::min<int64_t>(tiles, static_cast<int64_t>(sm_count()) * ctas_per_sm));
  cudaError_t e;
  switch (mode) {
    case DFC_MODE_PLAIN: e = launch_np<DFC_MODE_PLAIN>(b, grid, pdl, st); break;
    case DFC_MODE_SIGNFIBER: e = launch_np<DFC_MODE_SIGNFIBER>(b, grid, pdl, st); break;
    default: e = launch_np<DFC_MODE_PACKED>(b, grid, pdl, st); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_cuda_error(e);
    return DFC_ERR_CUDA;
  }
  return launch_status();
}

// ---- the switch's sums, read back ----------------------------------------
__global__ void __launch_bounds__(kThreads)
    multicast_sum_kernel(const uint16_t* mc, float* out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const int64_t n8 = n / kVec;
  for (int64_t k = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; k < n8; k += stride) {
    float g[8];
    nvls_sum8(mc + k * kVec, g);
    float4* o = reinterpret_cast<float4*>(out + k * kVec);
    o[0] = make_float4(g[0], g[1], g[2], g[3]);
    o[1] = make_float4(g[4], g[5], g[6], g[7]);
  }
  for (int64_t j = n8 * kVec + blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; j < n;
       j += stride)
    out[j] = nvls_sum1(mc, j);
}

// ---- barrier --------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct BarrierArgs {
  uint32_t* slots[kMaxPeers];  // every rank's signal array (n_peers words each)
  int32_t n_peers;
  int32_t rank;
  uint32_t epoch;
  int32_t* error;              // set to 1 + the peer waited for when the wait gives up
  uint64_t timeout_ns;
};

__global__ void peer_barrier_kernel(const __grid_constant__ BarrierArgs a) {
  // A programmatic dependent launched after this kernel (the fused step with
  // a compression in its grid) may start now; its step tiles still wait for
  // this grid to finish (griddepcontrol.wait), its compression tiles do not.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int q = threadIdx.x;
  if (q >= a.n_peers) return;
  // an earlier barrier gave up: signal nobody, wait for nobody
  if (*static_cast<volatile int32_t*>(a.error) != 0) return;
  __threadfence_system();  // this rank's earlier writes, local and remote, come first
  st_release_sys(a.slots[q] + a.rank, a.epoch);
  const uint32_t* mine = a.slots[a.rank] + q;
  const uint64_t start = globaltimer();
  while (static_cast<int32_t>(ld_acquire_sys(mine) - a.epoch) < 0) {
    if (globaltimer() - start > a.timeout_ns) {
      atomicExch(a.error, 1 + q);
      return;
    }
    __nanosleep(256);
  }
}

bool peers_ok(const void* const* ptrs, int32_t n) {
  for (int32_t q = 0; q < n; ++q)
    if (!ptrs[q]) return false;
  return true;
}

}  // namespace
}  // namespace dfc

namespace dfc {
namespace {

int fused_step(const void* const* comp_ptrs, void* const* param_ptrs, const void* comp_multicast,
               void* param_multicast, int32_t n_peers, int32_t rank,
               const DfcPeerSegment* segments, int32_t n_segments, const DfcHyper* hypers,
               int32_t n_hypers, int32_t mode, const float* device_grad_scale,
               const int32_t* error_flag, const DfcCompressRange* next, uint32_t flags,
               int32_t ctas_per_sm, cudaStream_t st) {
  if (n_peers < 1 || n_peers > kMaxPeers || rank < 0 || rank >= n_peers) return DFC_ERR_SIZE;
  if (n_segments < 0 || n_hypers < 0) return DFC_ERR_SIZE;
  if (mode != DFC_MODE_PLAIN && mode != DFC_MODE_SIGNFIBER && mode != DFC_MODE_PACKED)
    return DFC_ERR_MODE;
  if (flags & ~static_cast<uint32_t>(DFC_FUSED_AFTER_BARRIER)) return DFC_ERR_MODE;
  bool pdl = (flags & DFC_FUSED_AFTER_BARRIER) != 0;  // the first launch only
  const bool compress = next && next->numel != 0;
  if (compress) {
    if (next->numel < 0 || next->numel % 4 != 0) return DFC_ERR_SIZE;
    if (!next->grad || !next->comp || !next->resid) return DFC_ERR_NULL;
    if (!aligned(next->grad, 16) || !aligned(next->comp, 8) || !aligned(next->resid, 8))
      return DFC_ERR_ALIGN;
    if ((next->numel / 4 + 2 * kThreads - 1) / (2 * kThreads) > INT32_MAX / 2) return DFC_ERR_SIZE;
  }
  if (n_segments == 0 && !compress) return DFC_OK;
  if (!comp_ptrs || !param_ptrs || (!segments && n_segments > 0) || (!hypers && n_hypers > 0))
    return DFC_ERR_NULL;
  if (!peers_ok(comp_ptrs, n_peers) || !peers_ok(param_ptrs, n_peers)) return DFC_ERR_NULL;
  for (int32_t q = 0; q < n_peers; ++q)
    if (!aligned(comp_ptrs[q], 16) || !aligned(param_ptrs[q], 16)) return DFC_ERR_ALIGN;
  if ((comp_multicast == nullptr) != (param_multicast == nullptr)) return DFC_ERR_NULL;
  if (!aligned(comp_multicast, 16) || !aligned(param_multicast, 16)) return DFC_ERR_ALIGN;
  if (!aligned(error_flag, 4)) return DFC_ERR_ALIGN;
  for (int32_t i = 0; i < n_segments; ++i) {
    const DfcPeerSegment& s = segments[i];
    if (s.numel < 0 || s.offset < 0) return DFC_ERR_SIZE;
    if (s.numel == 0) continue;
    if (!s.exp_avg || !s.exp_avg_sq) return DFC_ERR_NULL;
    if (!aligned(s.exp_avg, 4) || !aligned(s.exp_avg_sq, 4)) return DFC_ERR_ALIGN;
    if (s.hyper < 0 || s.hyper >= n_hypers) return DFC_ERR_HYPER;
    if ((s.numel + kTile - 1) / kTile > INT32_MAX / 2) return DFC_ERR_SIZE;
  }
  ZeroBatch<kMaxSegs, kMaxHypers> b;
  for (int32_t q = 0; q < kMaxPeers; ++q) {
    b.comp[q] = q < n_peers ? static_cast<const uint16_t*>(comp_ptrs[q]) : nullptr;
    b.param[q] = q < n_peers ? static_cast<float*>(param_ptrs[q]) : nullptr;
  }
  b.comp_mc = static_cast<const uint16_t*>(comp_multicast);
  b.param_mc = static_cast<float*>(param_multicast);
  b.dev_scale = device_grad_scale;
  b.error = error_flag;
  b.n_peers = n_peers;
  b.rank = rank;
  // the compression rides with the first launch only
  b.cgrad = compress ? next->grad : nullptr;
  b.ccomp = compress ? next->comp : nullptr;
  b.cresid = compress ? next->resid : nullptr;
  b.cquads = compress ? next->numel / 4 : 0;
  b.ctiles = compress ? static_cast<int32_t>((b.cquads + 2 * kThreads - 1) / (2 * kThreads)) : 0;
  std::vector<int32_t> local(static_cast<size_t>(n_hypers), -1);
  std::vector<int32_t> used;
  auto reset = [&]() {
    for (int32_t g : used) local[g] = -1;
    used.clear();
    b.n_segs = 0;
    b.tile_base[0] = 0;
  };
  reset();
  for (int32_t i = 0; i < n_segments; ++i) {
    const DfcPeerSegment& s = segments[i];
    if (s.numel == 0) continue;
    const int32_t tiles = static_cast<int32_t>((s.numel + kTile - 1) / kTile);
    const bool need = local[s.hyper] < 0;
    if (b.n_segs == kMaxSegs || (need && static_cast<int>(used.size()) == kMaxHypers) ||
        b.tile_base[b.n_segs] > INT32_MAX / 2 - tiles) {
      const int rc = launch(b, mode, ctas_per_sm, pdl, st);
      if (rc != DFC_OK) return rc;
      reset();
      b.ctiles = 0;
      pdl = false;
    }
    if (local[s.hyper] < 0) {
      local[s.hyper] = static_cast<int32_t>(used.size());
      b.hyper[used.size()] = hypers[s.hyper];
      used.push_back(s.hyper);
    }
    PeerSegArg& a = b.seg[b.n_segs];
    a.offset = s.offset;
    a.n = s.numel;
    a.m = s.exp_avg;
    a.v = s.exp_avg_sq;
    a.hyper = local[s.hyper];
    a.vec = (s.offset % 4 == 0) && aligned(s.exp_avg, 16) && aligned(s.exp_avg_sq, 16);
    b.tile_base[b.n_segs + 1] = b.tile_base[b.n_segs] + tiles;
    ++b.n_segs;
  }
  return (b.n_segs || b.ctiles) ? launch(b, mode, ctas_per_sm, pdl, st) : DFC_OK;
}

}  // namespace
}  // namespace dfc

extern "C" int dfc_zero_fused_step(const void* const* comp_ptrs, void* const* param_ptrs,
                                   const void* comp_multicast, void* param_multicast,
                                   int32_t n_peers, int32_t rank, const DfcPeerSegment* segments,
                                   int32_t n_segments, const DfcHyper* hypers, int32_t n_hypers,
                                   int32_t mode, const float* device_grad_scale,
                                   const int32_t* error_flag, int32_t ctas_per_sm, void* stream) {
  return dfc::fused_step(comp_ptrs, param_ptrs, comp_multicast, param_multicast, n_peers, rank,
                         segments, n_segments, hypers, n_hypers, mode, device_grad_scale,
                         error_flag, nullptr, 0, ctas_per_sm, static_cast<cudaStream_t>(stream));
}

extern "C" int dfc_zero_fused_step_ef(const void* const* comp_ptrs, void* const* param_ptrs,
                                      const void* comp_multicast, void* param_multicast,
                                      int32_t n_peers, int32_t rank,
                                      const DfcPeerSegment* segments, int32_t n_segments,
                                      const DfcHyper* hypers, int32_t n_hypers, int32_t mode,
                                      const float* device_grad_scale, const int32_t* error_flag,
                                      const DfcCompressRange* next, uint32_t flags,
                                      int32_t ctas_per_sm, void* stream) {
  return dfc::fused_step(comp_ptrs, param_ptrs, comp_multicast, param_multicast, n_peers, rank,
                         segments, n_segments, hypers, n_hypers, mode, device_grad_scale,
                         error_flag, next, flags, ctas_per_sm, static_cast<cudaStream_t>(stream));
}

extern "C" int dfc_multicast_sum_bf16(const void* comp_multicast, float* out, int64_t numel,
                                      void* stream) {
  using namespace dfc;
  if (numel < 0) return DFC_ERR_SIZE;
  if (numel == 0) return DFC_OK;
  if (!comp_multicast || !out) return DFC_ERR_NULL;
  if (!aligned(comp_multicast, 16) || !aligned(out, 16)) return DFC_ERR_ALIGN;
  const int64_t blocks = std::min<int64_t>((numel / kVec + kThreads - 1) / kThreads + 1,
                                           resident_ctas(multicast_sum_kernel, kThreads));
  multicast_sum_kernel<<<static_cast<int>(blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(comp_multicast), out, numel);
  return launch_status();
}

extern "C" int dfc_peer_barrier(uint32_t* const* slot_ptrs, int32_t n_peers, int32_t rank,
                                uint32_t epoch, int32_t* error_flag, int64_t timeout_ns,
                                void* stream) {
  using namespace dfc;
  if (n_peers < 1 || n_peers > kMaxPeers || rank < 0 || rank >= n_peers || timeout_ns <= 0)
    return DFC_ERR_SIZE;
  if (!slot_ptrs || !error_flag || !peers_ok(reinterpret_cast<const void* const*>(slot_ptrs), n_peers))
    return DFC_ERR_NULL;
  for (int32_t q = 0; q < n_peers; ++q)
    if (!aligned(slot_ptrs[q], 4)) return DFC_ERR_ALIGN;
  if (!aligned(error_flag, 4)) return DFC_ERR_ALIGN;
  BarrierArgs a;
  for (int32_t q = 0; q < kMaxPeers; ++q) a.slots[q] = q < n_peers ? slot_ptrs[q] : nullptr;
  a.n_peers = n_peers;
  a.rank = rank;
  a.epoch = epoch;
  a.error = error_flag;
  a.timeout_ns = static_cast<uint64_t>(timeout_ns);
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}
