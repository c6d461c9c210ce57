// Sign-fiber payload I/O on the device: bit 31 of every second-moment word,
// concatenated over a list of word ranges, read into or written from a
// little-endian packed byte buffer (remote/torch_fiber.py:120-185).
//
// Each warp owns one span of 512 consecutive payload bits (= words); a CTA of
// 8 warps owns 4096, and the grid has one CTA per 4096 bits, dispatched in
// address order, so the accesses in flight stay in one compact window of
// the words (a persistent grid-stride form measured 0.78 of the copy
// bandwidth on reads; its warps drift apart over the whole buffer).
//
// Vector path -- the span lies in one range, its first word is 16-byte
// aligned and the payload pointer 4-byte aligned: lane l moves words
// 128 j + 4 l .. + 3 of group j (j = 0..3) as one 16-byte access.  Those
// four words are payload bits 4 l .. 4 l + 3 of the group's 128, i.e. nibble
// (l & 7) of the group's 32-bit payload word l >> 3 (little-endian bit
// order).  A read forms each lane's nibble, ORs the 8 nibbles of a 32-bit
// payload word together with three butterfly shuffles and stores it from
// one lane; a write loads the payload word and rewrites bit 31 of its four
// words.  Writes never race: every word belongs to one lane, and every
// payload word to one 8-lane group.
// Per-word path -- a span at a range boundary, at the end of the payload, or
// misaligned: one lane per word, 32-word groups, a ballot gathers the group's
// 4 payload bytes on a read; each lane looks its range up.
// Holes -- a range with no words (NULL) stands for bits that live elsewhere
// (another rank's pieces of a ZeRO-1 fiber): they read as zero and are left
// alone by a write.
// The range list lives in launch parameters (up to kMaxRanges per launch); a
// call with more ranges is split into launches at byte boundaries of the
// payload.
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

constexpr int kSpan = 512;               // payload bits (words) per warp
constexpr int kVecGroups = kSpan / 128;  // 16-byte accesses per lane
constexpr int kWordGroups = 8;           // 32-word groups per per-word pass
constexpr int kCtaSpan = kSpan * (kThreads / 32);

// Bits [k0, k0 + 32 * kWordGroups) of the launch, one lane per word; r is a
// range holding bit first_bit + k0 or an earlier one (ranges ascend).
template <bool WRITE>
__device__ __forceinline__ void span_by_word(const FiberBatch& b, uint8_t* bytes, int64_t k0,
                                             int r, int lane) {
  const int64_t nbytes = (b.n_bits + 7) / 8;
  uint32_t* ptr[kWordGroups];
#pragma unroll
  for (int j = 0; j < kWordGroups; ++j) {
    const int64_t k = k0 + 32 * j + lane;
    ptr[j] = nullptr;
    if (k < b.n_bits) {
      const int64_t g = b.first_bit + k;
      while (g >= b.range_base[r + 1]) ++r;
      ptr[j] = b.words[r] ? b.words[r] + (g - b.range_base[r]) : nullptr;  // a hole: none
    }
  }
  uint32_t word[kWordGroups], in[kWordGroups];
  // every load before the first store: a byte load after a word store could
  // alias it as far as the compiler knows, and would wait for it
#pragma unroll
  for (int j = 0; j < kWordGroups; ++j) {
    word[j] = ptr[j] ? *ptr[j] : 0u;
    in[j] = (WRITE && ptr[j]) ? bytes[(k0 + 32 * j + lane) >> 3] : 0u;
  }
#pragma unroll
  for (int j = 0; j < kWordGroups; ++j) {
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

template <bool WRITE>
__global__ void __launch_bounds__(kThreads) fiber_kernel(const __grid_constant__ FiberBatch b,
                                                         uint8_t* bytes, int32_t payload_vec) {
  const int lane = threadIdx.x & 31;
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * kCtaSpan + (threadIdx.x >> 5) * kSpan;
  if (k0 >= b.n_bits) return;  // warp-uniform
  const int r = find_range(b, b.first_bit + k0);
  const int64_t off = b.first_bit + k0 - b.range_base[r];
  const bool whole = k0 + kSpan <= b.n_bits && b.first_bit + k0 + kSpan <= b.range_base[r + 1];
  if (whole && b.words[r] == nullptr) {  // the span lies in a hole
    if (!WRITE) {
      const int64_t byte0 = k0 / 8;
      for (int k = lane; k < kSpan / 8; k += 32) bytes[byte0 + k] = 0;
    }
    return;
  }
  uint32_t* base = b.words[r] ? b.words[r] + off : nullptr;
  if (payload_vec && whole && (reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
    uint4* w4 = reinterpret_cast<uint4*>(base) + lane;
    uint32_t* pw = reinterpret_cast<uint32_t*>(bytes) + k0 / 32 + (lane >> 3);
    const int shift = 4 * (lane & 7);
    uint4 W[kVecGroups];
#pragma unroll
    for (int j = 0; j < kVecGroups; ++j) W[j] = __ldcs(w4 + 32 * j);
    if (WRITE) {
      uint32_t P[kVecGroups];
#pragma unroll
      for (int j = 0; j < kVecGroups; ++j) P[j] = pw[4 * j];
#pragma unroll
      for (int j = 0; j < kVecGroups; ++j) {
        const uint32_t nib = P[j] >> shift;
        W[j].x = (W[j].x & 0x7FFFFFFFu) | (nib << 31);
        W[j].y = (W[j].y & 0x7FFFFFFFu) | ((nib >> 1) << 31);
        W[j].z = (W[j].z & 0x7FFFFFFFu) | ((nib >> 2) << 31);
        W[j].w = (W[j].w & 0x7FFFFFFFu) | ((nib >> 3) << 31);
        __stcs(w4 + 32 * j, W[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < kVecGroups; ++j) {
        uint32_t v = ((W[j].x >> 31) | ((W[j].y >> 31) << 1) | ((W[j].z >> 31) << 2) |
                      ((W[j].w >> 31) << 3)) << shift;
        v |= __shfl_xor_sync(0xFFFFFFFFu, v, 1);
        v |= __shfl_xor_sync(0xFFFFFFFFu, v, 2);
        v |= __shfl_xor_sync(0xFFFFFFFFu, v, 4);
        if ((lane & 7) == 0) pw[4 * j] = v;
      }
    }
    return;
  }
#pragma unroll 1
  for (int h = 0; h < kSpan / (32 * kWordGroups); ++h)
    span_by_word<WRITE>(b, bytes, k0 + 32 * kWordGroups * h, r, lane);
}

template <bool WRITE>
int fiber_call(const DfcWordRange* ranges, int32_t n_ranges, int64_t start_bit, int64_t n_bits,
               uint8_t* bytes, cudaStream_t st) {
  if (n_ranges < 0 || start_bit < 0 || n_bits < 0) return n_ranges < 0 ? DFC_ERR_SIZE : DFC_ERR_RANGE;
  if (n_ranges > 0 && !ranges) return DFC_ERR_NULL;
  int64_t total = 0;
  for (int32_t i = 0; i < n_ranges; ++i) {
    if (ranges[i].count < 0) return DFC_ERR_SIZE;
    // a NULL words pointer is a hole: bits that live elsewhere
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
    const int64_t ctas = (b.n_bits + kCtaSpan - 1) / kCtaSpan;
    if (ctas > INT32_MAX) return DFC_ERR_SIZE;
    uint8_t* launch_bytes = bytes + done / 8;
    fiber_kernel<WRITE><<<static_cast<unsigned>(ctas), kThreads, 0, st>>>(
        b, launch_bytes, aligned(launch_bytes, 4) ? 1 : 0);
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
