// Sign-fiber payload I/O on the device: bit 31 of every second-moment word,
// concatenated over a list of word ranges, read into or written from a
// little-endian packed byte buffer (remote/torch_fiber.py:120-185).  One lane
// per word, so a warp's word accesses are coalesced: a read gathers the 32
// lanes' bits with __ballot_sync into 4 payload bytes (bit j of the mask is
// lane j's bit, which is the little-endian bit order of the payload); a
// write reads its bit from the payload byte and rewrites its own word, so
// writes never race.  Each warp takes kGroups groups of 32 words per
// iteration, with every group's word load issued before the first use.  The
// range list lives in launch parameters (up to kMaxRanges per launch); a call
// with more ranges is split into launches at byte boundaries of the payload.
#include <algorithm>

#include "dfc_common.cuh"

namespace dfc {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxRanges = 1300;

struct FiberBatch {
  int32_t n_ranges;
  int32_t pad;
  int64_t first_bit;   // global fiber bit of this launch's byte 0 (byte aligned in the payload)
  int64_t n_bits;      // bits this launch reads/writes, starting at first_bit
  int64_t range_base[kMaxRanges + 1];  // global fiber bit of each range's word 0
  uint32_t* words[kMaxRanges];
};
static_assert(sizeof(FiberBatch) <= 32000, "launch parameter limit");

__device__ __forceinline__ int find_range(const FiberBatch& b, int64_t g) {
  int lo = 0, hi = b.n_ranges;  // range_base[lo] <= g < range_base[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (b.range_base[mid] <= g) lo = mid; else hi = mid;
  }
  return lo;
}

constexpr int kGroups = 8;  // 32-word groups per warp per iteration

template <bool WRITE>
__global__ void __launch_bounds__(kThreads) fiber_kernel(const __grid_constant__ FiberBatch b,
                                                         uint8_t* bytes) {
  const int lane = threadIdx.x & 31;
  const int64_t nbytes = (b.n_bits + 7) / 8;
  const int64_t span = 32 * kGroups;  // payload bits per warp iteration
  const int64_t n_iter = (b.n_bits + span - 1) / span;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
       w < n_iter; w += warps) {
    const int64_t k0 = span * w;  // first payload bit of this iteration (warp-uniform)
    int r = find_range(b, b.first_bit + k0);
    if (k0 + span <= b.n_bits && b.first_bit + k0 + span <= b.range_base[r + 1]) {
      // The whole iteration lies in range r (the common case): one base
      // pointer, and word (32 j + lane) of it for group j -- no per-word
      // index arithmetic.  k0 + 32 j is a multiple of 8, so lane's payload
      // bit is bit (lane & 7) of byte (k0 + 32 j + lane) / 8.
      uint32_t* base = b.words[r] + (b.first_bit + k0 - b.range_base[r]) + lane;
      uint32_t word[kGroups], in[kGroups];
#pragma unroll
      for (int j = 0; j < kGroups; ++j) word[j] = base[32 * j];
      // every load before the first store: a byte load after a word store
      // could alias it as far as the compiler knows, and would wait for it
      if (WRITE) {
#pragma unroll
        for (int j = 0; j < kGroups; ++j) in[j] = bytes[(k0 + 32 * j + lane) >> 3];
      }
#pragma unroll
      for (int j = 0; j < kGroups; ++j) {
        if (WRITE) {
          base[32 * j] = (word[j] & 0x7FFFFFFFu) | (((in[j] >> (lane & 7)) & 1u) << 31);
        } else {
          const uint32_t mask = __ballot_sync(0xFFFFFFFFu, (word[j] >> 31) != 0u);
          if (lane < 4) bytes[(k0 + 32 * j) / 8 + lane] = static_cast<uint8_t>(mask >> (8 * lane));
        }
      }
      continue;
    }
    // An iteration at a range boundary or at the end of the payload: each
    // lane finds its own range.
    uint32_t* ptr[kGroups];
    uint32_t word[kGroups];
#pragma unroll
    for (int j = 0; j < kGroups; ++j) {
      const int64_t k = k0 + 32 * j + lane;
      ptr[j] = nullptr;
      if (k < b.n_bits) {
        const int64_t g = b.first_bit + k;
        while (g >= b.range_base[r + 1]) ++r;  // ranges ascend with g
        ptr[j] = b.words[r] + (g - b.range_base[r]);
      }
    }
    uint32_t in[kGroups];
#pragma unroll
    for (int j = 0; j < kGroups; ++j) {
      word[j] = ptr[j] ? *ptr[j] : 0u;
      in[j] = (WRITE && ptr[j]) ? bytes[(k0 + 32 * j + lane) >> 3] : 0u;
    }
#pragma unroll
    for (int j = 0; j < kGroups; ++j) {
      const int64_t k = k0 + 32 * j + lane;
      if (WRITE) {
        if (ptr[j]) *ptr[j] = (word[j] & 0x7FFFFFFFu) | (((in[j] >> (k & 7)) & 1u) << 31);
      } else {
        const uint32_t mask = __ballot_sync(0xFFFFFFFFu, (word[j] >> 31) != 0u);
        const int64_t byte = (k0 + 32 * j) / 8 + lane;  // lanes 0..3: the group's 4 bytes
        if (lane < 4 && byte < nbytes) bytes[byte] = static_cast<uint8_t>(mask >> (8 * lane));
      }
    }
  }
}

template <bool WRITE>
int fiber_call(const DfcWordRange* ranges, int32_t n_ranges, int64_t start_bit, int64_t n_bits,
               uint8_t* bytes, cudaStream_t st) {
  if (n_ranges < 0 || start_bit < 0 || n_bits < 0) return n_ranges < 0 ? DFC_ERR_SIZE : DFC_ERR_RANGE;
  if (n_ranges > 0 && !ranges) return DFC_ERR_NULL;
  int64_t total = 0;
  for (int32_t i = 0; i < n_ranges; ++i) {
    if (ranges[i].count < 0) return DFC_ERR_SIZE;
    if (ranges[i].count > 0 && !ranges[i].words) return DFC_ERR_NULL;
    if (!aligned(ranges[i].words, 4)) return DFC_ERR_ALIGN;
    total += ranges[i].count;
  }
  if (start_bit > total || n_bits > total - start_bit) return DFC_ERR_RANGE;
  if (n_bits == 0) return DFC_OK;
  if (!bytes) return DFC_ERR_NULL;

  // Walk the ranges that intersect [start_bit, start_bit + n_bits) and cut
  // the payload into launches of at most kMaxRanges ranges, each starting on
  // a payload byte boundary so no two launches share a byte.
  FiberBatch b;
  int64_t pos = 0;        // global bit of range i's first word
  int32_t i = 0;
  while (i < n_ranges && pos + ranges[i].count <= start_bit) pos += ranges[i++].count;
  int64_t done = 0;       // payload bits handled so far
  while (done < n_bits) {
    const int64_t first = start_bit + done;
    // rewind to the range holding `first`
    while (pos + ranges[i].count <= first) pos += ranges[i++].count;
    b.n_ranges = 0;
    b.first_bit = first;
    int64_t p = pos;
    int32_t j = i;
    while (j < n_ranges && b.n_ranges < kMaxRanges && p < start_bit + n_bits) {
      if (ranges[j].count > 0) {
        b.range_base[b.n_ranges] = p;
        b.words[b.n_ranges] = ranges[j].words;
        ++b.n_ranges;
      }
      p += ranges[j].count;
      ++j;
    }
    b.range_base[b.n_ranges] = p;
    int64_t end = std::min<int64_t>(p, start_bit + n_bits);
    if (end < start_bit + n_bits) {
      // not the last launch: stop at the last whole payload byte
      const int64_t whole = ((end - first) / 8) * 8;
      end = first + whole;
      if (whole == 0) return DFC_ERR_SIZE;  // more than kMaxRanges ranges inside one byte
    }
    b.n_bits = end - first;
    const int64_t iters = (b.n_bits + 32 * kGroups - 1) / (32 * kGroups);  // warp iterations
    const int64_t want = (iters + kThreads / 32 - 1) / (kThreads / 32);
    const int grid = static_cast<int>(
        std::max<int64_t>(1, std::min<int64_t>(want, resident_ctas(fiber_kernel<WRITE>, kThreads))));
    fiber_kernel<WRITE><<<grid, kThreads, 0, st>>>(b, bytes + done / 8);
    const int rc = launch_status();
    if (rc != DFC_OK) return rc;
    done += b.n_bits;
  }
  return DFC_OK;
}

}  // namespace
}  // namespace dfc

extern "C" int dfc_fiber_read(const DfcWordRange* ranges, int32_t n_ranges, int64_t start_bit,
                              int64_t n_bits, uint8_t* bytes, void* stream) {
  return dfc::fiber_call<false>(ranges, n_ranges, start_bit, n_bits, bytes,
                                static_cast<cudaStream_t>(stream));
}

extern "C" int dfc_fiber_write(const DfcWordRange* ranges, int32_t n_ranges, int64_t start_bit,
                               int64_t n_bits, const uint8_t* bytes, void* stream) {
  return dfc::fiber_call<true>(ranges, n_ranges, start_bit, n_bits, const_cast<uint8_t*>(bytes),
                               static_cast<cudaStream_t>(stream));
}
