// Replay records of the sign-fiber continual-learning benchmark, encoded and
// decoded on the device in batches (remote/vision_benchmark.py:74-100,
// CIFAR4BitCodec).  A record is 1552 bytes:
//
//   [0, 4)       "CF4B"
//   [4, 6)       label, uint16 little-endian
//   [6, 8)       task, uint16 little-endian
//   [8, 1544)    3072 pixels quantised to 4 bits, q = clamp(rint(x * 15), 0, 15)
//                (nearest, ties to even; NaN -> 0), pixel 2i in the low nibble
//                of byte 8 + i and pixel 2i + 1 in the high nibble
//   [1544, 1548) CRC-32 (zlib: reflected polynomial 0xEDB88320, initial and
//                final value 0xFFFFFFFF) of bytes [0, 1544), little-endian
//   [1548, 1552) zero
//
// One warp per record, one CTA per 8 consecutive records, CTAs dispatched in
// address order (a persistent grid-stride form ran at 0.94 / 0.84 of the copy
// bandwidth for encode / decode, this one at 0.99 / 0.94).  The CRC tables
// are compile-time constants in device memory, copied into shared memory as
// a CTA starts.  The warp stages the record in shared memory with
// coalesced 16-byte loads or stores, and splits the CRC: lane k runs the
// table-driven CRC over its own 48-byte run of the record (lane 0 also over
// the 8-byte header, starting from 0xFFFFFFFF; the others from 0), then
// multiplies its remainder by x^(8 * bytes after its run) mod P and the warp
// XORs the 32 products.  That is the CRC of the whole record because the
// remainder is linear over GF(2):  R(A || B) = R(A) * x^(8|B|) + R(B).
#include <algorithm>
#include <mutex>

#include "dfc_common.cuh"

namespace dfc {
namespace {

constexpr int kRecordBytes = DFC_REPLAY_RECORD_BYTES;  // 1552
constexpr int kPixels = DFC_REPLAY_PIXELS;             // 3072
constexpr int kCrcBytes = 1544;                        // bytes covered by the CRC
constexpr int kHeader = 8;
constexpr int kRun = 48;                               // packed bytes per lane
constexpr int kWarps = 8;                              // records per CTA
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kPoly = 0xEDB88320u;                // reflected 0x04C11DB7
constexpr uint32_t kOne = 0x80000000u;                 // x^0, reflected

static_assert(kHeader + 32 * kRun == kCrcBytes, "record layout");
static_assert(kRecordBytes % 16 == 0, "records are 16-byte aligned");

// a * b mod P, both in the reflected representation (bit 31 holds x^0):
// the sum over the set coefficients a_i of b * x^i, with b * x^(i+1)
// obtained from b * x^i by one shift and a conditional reduction.
__host__ __device__ inline uint32_t gf2_mulmod(uint32_t a, uint32_t b) {
  uint32_t p = 0;
  for (int i = 0; i < 32; ++i) {
    if (a & (kOne >> i)) p ^= b;
    b = (b >> 1) ^ ((b & 1u) ? kPoly : 0u);
  }
  return p;
}

// x^(8 n) mod P by square-and-multiply.
uint32_t x_pow_8n(uint64_t n) {
  uint32_t result = kOne, base = kOne >> 8;  // x^8
  while (n) {
    if (n & 1) result = gf2_mulmod(result, base);
    base = gf2_mulmod(base, base);
    n >>= 1;
  }
  return result;
}

struct Shifts {
  uint32_t lane[32];  // x^(8 * bytes after lane k's run) mod P
};

const Shifts& shifts() {
  static Shifts s;
  static std::once_flag once;
  std::call_once(once, [] {
    for (int k = 0; k < 32; ++k) s.lane[k] = x_pow_8n(static_cast<uint64_t>(kRun) * (31 - k));
  });
  return s;
}

// Slicing-by-4 tables: t[0][i] is the remainder of byte i shifted through
// eight steps of the reflected polynomial division; t[k][i] is that of byte
// i followed by k zero bytes, t[k][i] = (t[k-1][i] >> 8) ^ t[0][t[k-1][i] & 0xFF].
// A 32-bit word x = c ^ (4 message bytes) then advances the remainder with
// four independent lookups: t[3][x0] ^ t[2][x1] ^ t[1][x2] ^ t[0][x3].
struct CrcTables {
  uint32_t t[4][256];
};

constexpr CrcTables make_crc_tables() {
  CrcTables r{};
  for (int i = 0; i < 256; ++i) {
    uint32_t c = static_cast<uint32_t>(i);
    for (int k = 0; k < 8; ++k) c = (c >> 1) ^ ((c & 1u) ? kPoly : 0u);
    r.t[0][i] = c;
  }
  for (int k = 1; k < 4; ++k)
    for (int i = 0; i < 256; ++i) r.t[k][i] = (r.t[k - 1][i] >> 8) ^ r.t[0][r.t[k - 1][i] & 0xFFu];
  return r;
}

// Constant data of the library, fixed at compile time (no allocation).
__device__ const CrcTables g_crc_tables = make_crc_tables();

__device__ __forceinline__ void load_tables(uint32_t (*t)[256]) {
  for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) t[i >> 8][i & 255] = g_crc_tables.t[i >> 8][i & 255];
  __syncthreads();
}

// CRC-32 of the record staged at rec (bytes [0, 1544)), all 32 lanes.
__device__ __forceinline__ uint32_t record_crc(const uint8_t* rec, const uint32_t (*t)[256],
                                               const Shifts& sh, int lane) {
  const int start = lane == 0 ? 0 : kHeader + kRun * lane;
  const int end = kHeader + kRun * (lane + 1);
  uint32_t c = lane == 0 ? 0xFFFFFFFFu : 0u;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(rec + start);
  for (int i = 0; i < (end - start) / 4; ++i) {
    const uint32_t x = c ^ w[i];
    c = t[3][x & 0xFFu] ^ t[2][(x >> 8) & 0xFFu] ^ t[1][(x >> 16) & 0xFFu] ^ t[0][x >> 24];
  }
  c = gf2_mulmod(c, sh.lane[lane]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) c ^= __shfl_xor_sync(0xFFFFFFFFu, c, off);
  return ~c;
}

// clamp(rint(x * 15), 0, 15): the conversion rounds to nearest even and
// saturates to [0, 2^32 - 1] with NaN -> 0; the min clamps the top.
__device__ __forceinline__ uint32_t quant4(float x) {
  uint32_t q;
  asm("cvt.rni.sat.u32.f32 %0, %1;" : "=r"(q) : "f"(__fmul_rn(x, 15.0f)));
  return min(q, 15u);
}

struct EncodeArgs {
  const float* images;  // n records of 3072 FP32, image_stride floats apart
  int64_t image_stride;
  const int32_t* labels;
  const int32_t* tasks;
  uint8_t* records;     // n records, record_stride bytes apart
  int64_t record_stride;
  int64_t n;
  Shifts sh;
};

// Warp w of CTA c encodes record 8 c + w.
__global__ void __launch_bounds__(kThreads) encode_kernel(const __grid_constant__ EncodeArgs a) {
  __shared__ uint32_t tables[4][256];
  __shared__ __align__(16) uint8_t stage[kWarps][kRecordBytes];
  load_tables(tables);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* rec = stage[warp];
  uint16_t* packed = reinterpret_cast<uint16_t*>(rec + kHeader);
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (r < a.n) {
    const float4* src = reinterpret_cast<const float4*>(a.images + r * a.image_stride);
#pragma unroll 4
    for (int i = lane; i < kPixels / 4; i += 32) {
      const float4 x = __ldg(src + i);
      packed[i] = static_cast<uint16_t>(quant4(x.x) | (quant4(x.y) << 4) | (quant4(x.z) << 8) |
                                        (quant4(x.w) << 12));
    }
    if (lane == 0) {
      const uint32_t y = static_cast<uint32_t>(a.labels[r]) & 0xFFFFu;
      const uint32_t t = static_cast<uint32_t>(a.tasks[r]) & 0xFFFFu;
      reinterpret_cast<uint32_t*>(rec)[0] = 0x42344643u;  // "CF4B"
      reinterpret_cast<uint32_t*>(rec)[1] = y | (t << 16);
    }
    __syncwarp();
    const uint32_t crc = record_crc(rec, tables, a.sh, lane);
    if (lane == 0) {
      reinterpret_cast<uint32_t*>(rec + kCrcBytes)[0] = crc;
      reinterpret_cast<uint32_t*>(rec + kCrcBytes)[1] = 0u;
    }
    __syncwarp();
    uint4* dst = reinterpret_cast<uint4*>(a.records + r * a.record_stride);
    const uint4* s4 = reinterpret_cast<const uint4*>(rec);
    for (int i = lane; i < kRecordBytes / 16; i += 32) dst[i] = s4[i];
  }
}

struct DecodeArgs {
  const uint8_t* records;
  int64_t record_stride;
  float* images;        // n * 3072 FP32, contiguous
  int32_t* labels;
  int32_t* tasks;
  int32_t* status;      // DFC_RECORD_*
  int64_t n;
  Shifts sh;
};

// q / 15 for a 4-bit q, correctly rounded (what the reference's
// q.astype(float32) / 15 gives): y = q * RN(1/15) is corrected by one
// residual step, e = fma(-15, y, q), y + e * RN(1/15).  With 16 possible
// inputs this is checked exhaustively (tests/test_replay_oracle.py) rather
// than argued; it replaces two shared-memory table lookups per 4 pixels,
// which held the decode at 0.84 of the copy bandwidth (MIO throttle).
__device__ __forceinline__ float nibble_over_15(uint32_t q) {
  const float r = 0.0666666701436042785644531f;  // RN(1/15) = 0x3D888889
  const float x = static_cast<float>(q);
  const float y = __fmul_rn(x, r);
  const float e = __fmaf_rn(-15.0f, y, x);
  return __fmaf_rn(e, r, y);
}

// Warp w of CTA c decodes record 8 c + w.
__global__ void __launch_bounds__(kThreads) decode_kernel(const __grid_constant__ DecodeArgs a) {
  __shared__ uint32_t tables[4][256];
  __shared__ __align__(16) uint8_t stage[kWarps][kRecordBytes];
  load_tables(tables);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* rec = stage[warp];
  uint4* s4 = reinterpret_cast<uint4*>(rec);
  const uint16_t* packed = reinterpret_cast<const uint16_t*>(rec + kHeader);
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (r < a.n) {
    const uint4* src = reinterpret_cast<const uint4*>(a.records + r * a.record_stride);
    for (int i = lane; i < kRecordBytes / 16; i += 32) s4[i] = __ldg(src + i);
    __syncwarp();
    // pixels first, so their stores drain while the CRC runs
    float4* dst = reinterpret_cast<float4*>(a.images + r * kPixels);
#pragma unroll 4
    for (int i = lane; i < kPixels / 4; i += 32) {
      const uint32_t b = packed[i];
      __stcs(dst + i, make_float4(nibble_over_15(b & 15u), nibble_over_15((b >> 4) & 15u),
                                  nibble_over_15((b >> 8) & 15u), nibble_over_15(b >> 12)));
    }
    const uint32_t crc = record_crc(rec, tables, a.sh, lane);
    if (lane == 0) {
      const uint32_t* w = reinterpret_cast<const uint32_t*>(rec);
      const uint32_t stored = reinterpret_cast<const uint32_t*>(rec + kCrcBytes)[0];
      a.labels[r] = static_cast<int32_t>(w[1] & 0xFFFFu);
      a.tasks[r] = static_cast<int32_t>(w[1] >> 16);
      a.status[r] = w[0] != 0x42344643u ? DFC_RECORD_BAD_MAGIC
                                        : (stored != crc ? DFC_RECORD_BAD_CRC : DFC_RECORD_OK);
    }
  }
}

// One CTA per 8 records.
int64_t grid_for(int64_t n) { return (n + kWarps - 1) / kWarps; }

}  // namespace
}  // namespace dfc

extern "C" int dfc_replay_encode(const float* images, int64_t image_stride, const int32_t* labels,
                                 const int32_t* tasks, int64_t n_records, uint8_t* records,
                                 int64_t record_stride, void* stream) {
  using namespace dfc;
  if (n_records < 0 || image_stride < kPixels || record_stride < kRecordBytes) return DFC_ERR_SIZE;
  if (n_records == 0) return DFC_OK;
  if (!images || !labels || !tasks || !records) return DFC_ERR_NULL;
  if (!aligned(images, 16) || image_stride % 4 != 0 || !aligned(records, 16) ||
      record_stride % 16 != 0 || !aligned(labels, 4) || !aligned(tasks, 4))
    return DFC_ERR_ALIGN;
  EncodeArgs a;
  a.images = images;
  a.image_stride = image_stride;
  a.labels = labels;
  a.tasks = tasks;
  a.records = records;
  a.record_stride = record_stride;
  a.n = n_records;
  a.sh = shifts();
  if (grid_for(n_records) > INT32_MAX) return DFC_ERR_SIZE;
  encode_kernel<<<static_cast<unsigned>(grid_for(n_records)), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

extern "C" int dfc_replay_decode(const uint8_t* records, int64_t record_stride, int64_t n_records,
                                 float* images, int32_t* labels, int32_t* tasks, int32_t* status,
                                 void* stream) {
  using namespace dfc;
  if (n_records < 0 || record_stride < kRecordBytes) return DFC_ERR_SIZE;
  if (n_records == 0) return DFC_OK;
  if (!records || !images || !labels || !tasks || !status) return DFC_ERR_NULL;
  if (!aligned(records, 16) || record_stride % 16 != 0 || !aligned(images, 16) ||
      !aligned(labels, 4) || !aligned(tasks, 4) || !aligned(status, 4))
    return DFC_ERR_ALIGN;
  DecodeArgs a;
  a.records = records;
  a.record_stride = record_stride;
  a.images = images;
  a.labels = labels;
  a.tasks = tasks;
  a.status = status;
  a.n = n_records;
  a.sh = shifts();
  if (grid_for(n_records) > INT32_MAX) return DFC_ERR_SIZE;
  decode_kernel<<<static_cast<unsigned>(grid_for(n_records)), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}
