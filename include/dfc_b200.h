/*
 * dfc_b200.h -- C ABI of the B200 (sm_100a) DFC-AdamW step library
 * (libdfc_b200.so).
 *
 * The reference (YellowJune/T3st) has no native layer: its optimizer step is
 * eager PyTorch (remote/torch_fiber.py:68-117) and an unwired Triton kernel
 * (remote/triton_dfc_adamw.py:24-101, one launch per tensor).  Each entry
 * point below names the reference code it replaces.
 *
 * Conventions
 *  - Every pointer inside a descriptor is a DEVICE pointer, except where a
 *    comment says "host".  Descriptor arrays themselves (DfcSegment,
 *    DfcHyper, DfcGradRef, DfcWordRange) are HOST arrays read during the call
 *    and copied into the kernel's launch parameters: the caller may reuse
 *    them as soon as the call returns.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call
 *    is asynchronous and stream-ordered; none synchronises the host.
 *  - Return value: DFC_OK (0) or a negative DFC_ERR_* code.  Nothing aborts,
 *    nothing allocates device memory, nothing is cached between calls --
 *    with one exception, dfc_grad_stats_noalloc: its scratch is a static
 *    device array of the library, and the array's address on each device is
 *    looked up once and kept (see its comment).
 *  - Every launch is sized from its arguments; a bad argument is reported
 *    before any launch (nothing is half-applied).
 */
#ifndef DFC_B200_H_
#define DFC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DFC_ABI_VERSION 3

/* Entry points are the library's only exported symbols (it is built with
 * -fvisibility=hidden). */
#if defined(__GNUC__)
#define DFC_API __attribute__((visibility("default")))
#else
#define DFC_API
#endif

/* ---- status codes ---- */
#define DFC_OK 0
#define DFC_ERR_NULL (-1)      /* required pointer is NULL */
#define DFC_ERR_ALIGN (-2)     /* pointer not aligned to its element size */
#define DFC_ERR_SIZE (-3)      /* negative, inconsistent or too large size */
#define DFC_ERR_DTYPE (-4)     /* unknown gradient element type */
#define DFC_ERR_MODE (-5)      /* unknown moment-word format */
#define DFC_ERR_HYPER (-6)     /* hyper-set index out of range */
#define DFC_ERR_CUDA (-7)      /* CUDA runtime error (see dfc_last_cuda_error) */
#define DFC_ERR_RANGE (-8)     /* bit range outside the fiber */
#define DFC_ERR_SCRATCH (-9)   /* scratch buffer too small */

/* ---- moment-word formats ---- */
/* FP32 moments, second moment used as stored (enable_fiber=False,
 * remote/torch_fiber.py:94-96, 106-107). */
#define DFC_MODE_PLAIN 0
/* FP32 moments, bit 31 of the second-moment word is an opaque payload bit
 * kept across the step (remote/torch_fiber.py:90-105). */
#define DFC_MODE_SIGNFIBER 1
/* Packed words: high 16 bits = moment rounded to the nearest bf16 (ties away
 * from zero), low 16 bits = signed residual in FP32 ulps, so that
 * fp32 = (hi << 16) + (int16)lo exactly; a NaN is stored as the canonical
 * word 0x7FC00000.  Bit 31 of the first moment is its sign; bit 31 of the
 * second moment is the payload bit.  No counterpart in the reference (it
 * stores FP32 moments). */
#define DFC_MODE_PACKED 2

/* ---- element types of parameters and gradients ---- */
#define DFC_DTYPE_F32 0
#define DFC_DTYPE_BF16 1
#define DFC_DTYPE_F16 2
#define DFC_GRAD_F32 DFC_DTYPE_F32
#define DFC_GRAD_BF16 DFC_DTYPE_BF16
#define DFC_GRAD_F16 DFC_DTYPE_F16

/* One contiguous run of elements updated by the step: a whole parameter, or
 * the part of one that falls in a shard.  bf16/fp16 parameters keep FP32
 * moments; their update is computed in FP32 and rounded once to the
 * parameter type, with m and den rounded to it first, as PyTorch does for
 * the reference's mul_/addcdiv_ (remote/torch_fiber.py:114-116).  48 bytes. */
typedef struct DfcSegment {
  void* param;           /* param_dtype elements, updated in place */
  const void* grad;      /* grad_dtype elements */
  uint32_t* exp_avg;     /* first-moment words, updated in place */
  uint32_t* exp_avg_sq;  /* second-moment words, updated in place */
  int64_t numel;
  int32_t hyper;         /* index into the call's DfcHyper array */
  int16_t grad_dtype;    /* DFC_DTYPE_* */
  int16_t param_dtype;   /* DFC_DTYPE_* */
} DfcSegment;

/* FP32 scalars of one (param group, step count) pair, each rounded once
 * from the double the reference computes (remote/torch_fiber.py:75-116):
 *   beta1, 1-beta1, beta2, 1-beta2, sqrt(1-beta2^step), eps,
 *   decay = 1 - lr*wd (1 when wd == 0), neg_step_size = -lr/(1-beta1^step),
 *   grad_scale multiplies the gradient first (1 = none).  48 bytes. */
typedef struct DfcHyper {
  float beta1;
  float one_minus_beta1;
  float beta2;
  float one_minus_beta2;
  float sqrt_bc2;
  float eps;
  float decay;
  float neg_step_size;
  float grad_scale;
  float reserved[3];
} DfcHyper;

/* A gradient buffer for the statistics kernels.  24 bytes. */
typedef struct DfcGradRef {
  const void* grad;
  int64_t numel;
  int32_t grad_dtype;
  int32_t reserved;
} DfcGradRef;

/* Per-buffer gradient statistics.  24 bytes. */
typedef struct DfcGradStats {
  double sumsq;        /* sum of g*g, accumulated in double */
  float amax;          /* max |g| over non-NaN elements */
  int32_t reserved;
  int64_t nonfinite;   /* number of Inf/NaN elements */
} DfcGradStats;

/* Replay records (remote/vision_benchmark.py:74-100, CIFAR4BitCodec). */
#define DFC_REPLAY_RECORD_BYTES 1552
#define DFC_REPLAY_PIXELS 3072
#define DFC_RECORD_OK 0          /* magic and CRC-32 match */
#define DFC_RECORD_BAD_MAGIC 1   /* first four bytes are not "CF4B" */
#define DFC_RECORD_BAD_CRC 2     /* stored CRC-32 differs from the computed one */

/* Most ranks a fused ZeRO-1 call can span. */
#define DFC_MAX_PEERS 8

/* One run of this rank's elements for dfc_zero_fused_step.  40 bytes. */
typedef struct DfcPeerSegment {
  int64_t offset;        /* flat element index into every rank's comp and param arrays */
  int64_t numel;
  uint32_t* exp_avg;     /* this rank's first-moment words for the run */
  uint32_t* exp_avg_sq;  /* this rank's second-moment words for the run */
  int32_t hyper;         /* index into the call's DfcHyper array */
  int32_t reserved;
} DfcPeerSegment;

/* A gradient range for dfc_compress_ef run inside another launch's grid
 * (dfc_zero_fused_step_ef).  32 bytes. */
typedef struct DfcCompressRange {
  const float* grad;     /* numel FP32 gradients, 16-byte aligned */
  uint16_t* comp;        /* numel bf16 halves, 8-byte aligned */
  uint16_t* resid;       /* numel residual halves, 8-byte aligned */
  int64_t numel;         /* a multiple of 4 */
} DfcCompressRange;

/* A run of second-moment words whose bit 31 forms part of the sign fiber.
 * words == NULL makes the run a hole of `count` bits that live elsewhere
 * (in a ZeRO-1 fiber: another rank's pieces): reads return zero bits there,
 * writes leave it alone. */
typedef struct DfcWordRange {
  uint32_t* words;
  int64_t count;
} DfcWordRange;

DFC_API int dfc_abi_version(void);
DFC_API const char* dfc_strerror(int status);
/* cudaError_t of the last DFC_ERR_CUDA returned on this host thread. */
DFC_API int dfc_last_cuda_error(void);

/*
 * Fused multi-tensor DFC-AdamW step over `n_segments` segments in one launch
 * (more launches only beyond the per-launch capacity, 560 segments or 32
 * hyper sets).  Replaces the per-parameter loop of DFCAdamW.step
 * (remote/torch_fiber.py:74-117) and the one-tensor Triton launcher
 * dfc_adamw_step (remote/triton_dfc_adamw.py:63-101).
 *
 * segments, hypers: host arrays.  mode: DFC_MODE_*.  device_grad_scale:
 * NULL, or a device float multiplied into every gradient after
 * hyper.grad_scale (a clip coefficient computed on the device).
 */
DFC_API int dfc_mt_step(const DfcSegment* segments, int32_t n_segments, const DfcHyper* hypers,
                int32_t n_hypers, int32_t mode, const float* device_grad_scale, void* stream);

/*
 * Convert moment words between the reference's FP32 layout and the packed
 * layout, in place, over `n` words (no counterpart in the reference).
 * second != 0: bit 31 is the payload bit and is kept.
 * dfc_pack_moments: FP32 word -> packed word; dfc_unpack_moments: inverse.
 */
DFC_API int dfc_pack_moments(uint32_t* words, int64_t n, int32_t second, void* stream);
DFC_API int dfc_unpack_moments(uint32_t* words, int64_t n, int32_t second, void* stream);

/*
 * bf16 gradient compression with per-element error feedback over a flat
 * buffer (no counterpart in the reference, which keeps FP32 gradients,
 * remote/torch_fiber.py:83).  s = grad + e, where e is the residual left by
 * the previous call and recovered exactly from (comp, resid); comp <- s
 * rounded to the nearest bf16 (ties away from zero); resid <- the signed
 * 16-bit residual field.  comp and resid are read and written in place;
 * both start at zero.  ctas_per_sm <= 0: one CTA per 2048-element tile, for
 * a call that has the GPU to itself; 1..8: a persistent grid of at most that
 * many 256-thread CTAs per SM, leaving room for a kernel that runs beside it
 * on another stream (the ZeRO-1 pipeline's fused step).
 */
DFC_API int dfc_compress_ef(const float* grad, uint16_t* comp, uint16_t* resid, int64_t n,
                            int32_t ctas_per_sm, void* stream);

/*
 * Per-buffer gradient statistics with warp-shuffle block reductions and a
 * fixed-order second pass (deterministic).  `out` receives n_grads records
 * (device).  `scratch` (device) must hold dfc_grad_stats_scratch_bytes()
 * bytes.  No counterpart in the reference (it computes no statistics).
 */
DFC_API size_t dfc_grad_stats_scratch_bytes(const DfcGradRef* grads, int32_t n_grads);
DFC_API int dfc_grad_stats(const DfcGradRef* grads, int32_t n_grads, DfcGradStats* out, void* scratch,
                   size_t scratch_bytes, void* stream);

/*
 * dfc_grad_stats for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Same records, same kernels and the same
 * results as dfc_grad_stats, but the per-tile partial records live in a
 * device array inside the library instead of a caller-provided scratch
 * buffer, so the call needs nothing but the gradients and `out`.  It exists
 * for callers that cannot call cudaMalloc or any allocating routine when
 * they need the statistics (a host runtime whose device memory is all in
 * its own pool, a plugin whose host forbids device allocations during a
 * step).
 * Limit: a call may need at most DFC_GRAD_STATS_STATIC_RECORDS partial
 * records (one per 8192 elements of each buffer, at least one per buffer);
 * a larger request returns DFC_ERR_SCRATCH and launches nothing.  The array
 * (1.5 MiB) is held on every GPU that loads the library until exit.  The
 * first call on a device, with that device current, looks up the array's
 * device address; make that first call before any stream capture.  All
 * calls share the array: calls whose kernels overlap on the GPU race, so
 * order them on one stream.
 */
#define DFC_GRAD_STATS_STATIC_RECORDS 65536
DFC_API int dfc_grad_stats_noalloc(const DfcGradRef* grads, int32_t n_grads, DfcGradStats* out,
                                   void* stream);

/*
 * Global-norm clip coefficient from statistics records, on the device:
 * total = sqrt(sum sumsq); coef = min(1, max_norm / (total + 1e-6)).
 * Writes the coefficient to out_coef[0] and the norm to out_norm[0] (either
 * may be NULL).  Feeds dfc_mt_step's device_grad_scale.
 */
DFC_API int dfc_clip_coef(const DfcGradStats* stats, int32_t n_stats, float max_norm, float* out_coef,
                  float* out_norm, void* stream);

/*
 * Sign-fiber payload I/O on the device.  The fiber is the concatenation of
 * bit 31 of every word of the ranges, in order (remote/torch_fiber.py:
 * 120-185, TorchSignFiberChannel).  Bits [start_bit, start_bit + n_bits)
 * are read into / written from `bytes` (device, ceil(n_bits/8) bytes),
 * packed 8 per byte, least-significant bit first
 * (np.packbits(bitorder="little"), remote/torch_fiber.py:178, 184).  A read
 * leaves the unused high bits of the last byte zero; a write consumes
 * exactly n_bits bits.  Only bit 31 of each word is touched.  Ranges with
 * NULL words are holes (zero bits on a read, untouched on a write): with the
 * other ranks' runs as holes, a ZeRO-1 rank reads or writes its own bits of
 * the global fiber at their global positions, and a sum of the ranks' read
 * buffers is the whole fiber.  (The reference's channel,
 * remote/torch_fiber.py:151-185, addresses one process's tensors; holes
 * carry the same bit order across every rank's shard.)
 */
DFC_API int dfc_fiber_read(const DfcWordRange* ranges, int32_t n_ranges, int64_t start_bit,
                   int64_t n_bits, uint8_t* bytes, void* stream);
DFC_API int dfc_fiber_write(const DfcWordRange* ranges, int32_t n_ranges, int64_t start_bit,
                    int64_t n_bits, const uint8_t* bytes, void* stream);

/*
 * Replay-record codec on the device, one warp per record (replaces the
 * per-record host codec CIFAR4BitCodec.encode / .decode,
 * remote/vision_benchmark.py:79-100).  Record layout: "CF4B", label and task
 * as uint16 little-endian, 3072 pixels quantised to 4 bits as
 * clamp(round_half_even(x * 15), 0, 15) (NaN -> 0), two per byte with the
 * even pixel in the low nibble, the zlib CRC-32 of bytes [0, 1544)
 * little-endian, four zero bytes.
 *
 * dfc_replay_encode: images (device FP32, 16-byte aligned, image_stride
 * floats between records, a multiple of 4 and >= 3072), labels and tasks
 * (device int32; the low 16 bits are stored) -> records (device, 16-byte
 * aligned, record_stride bytes apart, a multiple of 16 and >= 1552).
 * dfc_replay_decode: records -> images (device FP32, contiguous, q / 15),
 * labels, tasks and status (device int32, DFC_RECORD_*).  Every record is
 * decoded whatever its status; the caller checks status.
 */
DFC_API int dfc_replay_encode(const float* images, int64_t image_stride, const int32_t* labels,
                              const int32_t* tasks, int64_t n_records, uint8_t* records,
                              int64_t record_stride, void* stream);
DFC_API int dfc_replay_decode(const uint8_t* records, int64_t record_stride, int64_t n_records,
                              float* images, int32_t* labels, int32_t* tasks, int32_t* status,
                              void* stream);

/*
 * ZeRO-1 shard step fused with its collectives over NVLink peer memory (no
 * counterpart in the reference, which has no distributed code; replaces
 * NCCL reduce-scatter + dfc_mt_step + NCCL all-gather).  comp_ptrs and
 * param_ptrs are host arrays of n_peers DEVICE addresses, indexed by rank, of
 * every rank's bf16 compressed gradients and flat FP32 parameters, all
 * mapped into this process (symmetric memory); 16-byte aligned.  For every
 * element j of the segments: g = comp_0[j] + comp_1[j] + ... (FP32, rank
 * order), the DFC-AdamW step on this rank's moment words, then the new
 * parameter stored to param_q[j] of every rank q.
 * comp_multicast, param_multicast: NULL, or the NVLink-multicast (NVSwitch)
 * addresses of the same two buffers; then the switch does the reduction
 * (multimem.ld_reduce, FP32 accumulation, result rounded to bf16 by the
 * switch) and the broadcast (multimem.st), for every element;
 * dfc_multicast_sum_bf16 returns the g values the switch produces.
 * The caller brackets the call with dfc_peer_barrier: before it so every
 * rank's gradients are complete, after it so every rank's parameters are.
 * ctas_per_sm <= 0: one CTA per 2048-element tile; > 0: a persistent grid of
 * at most that many CTAs per SM, so that the next bucket's dfc_compress_ef
 * (with its own cap) runs beside it instead of after it.
 * error_flag: NULL, or the device int that dfc_peer_barrier sets when it
 * gives up.  When it is non-zero as the kernel starts, the kernel returns
 * without a single load or store: after a barrier time-out no rank reads a
 * peer's half-written gradients or writes into a stalled peer's parameters,
 * and this rank's parameters and moments stay as they were.
 */
DFC_API int dfc_zero_fused_step(const void* const* comp_ptrs, void* const* param_ptrs,
                                const void* comp_multicast, void* param_multicast,
                                int32_t n_peers, int32_t rank, const DfcPeerSegment* segments,
                                int32_t n_segments, const DfcHyper* hypers, int32_t n_hypers,
                                int32_t mode, const float* device_grad_scale,
                                const int32_t* error_flag, int32_t ctas_per_sm, void* stream);

/*
 * dfc_zero_fused_step and dfc_compress_ef(next->grad, next->comp, next->resid,
 * next->numel) in one launch (no reference counterpart).  The grid's tiles are
 * the step's and the compression's, spread evenly, so the step's NVLink
 * traffic and the compression's HBM traffic overlap inside one kernel -- in
 * the ZeRO-1 pipeline, the compression of bucket b+1 beside the step of
 * bucket b.  Results are bit for bit those of the two calls.  next's buffers
 * must not overlap anything the step reads or writes.  The compression runs
 * even when *error_flag is set (it touches only the memory it is given).
 * next == NULL or next->numel == 0: dfc_zero_fused_step.
 * flags: 0, or DFC_FUSED_AFTER_BARRIER when the previous operation on the
 * stream is a dfc_peer_barrier: the grid is then launched as its
 * programmatic dependent, so the compression tiles run while the barrier
 * still waits, and the step tiles wait for the barrier to finish.  With that
 * flag next's buffers must already be complete before the barrier starts.
 * Other flag bits: DFC_ERR_MODE.
 */
#define DFC_FUSED_AFTER_BARRIER 1u
DFC_API int dfc_zero_fused_step_ef(const void* const* comp_ptrs, void* const* param_ptrs,
                                   const void* comp_multicast, void* param_multicast,
                                   int32_t n_peers, int32_t rank, const DfcPeerSegment* segments,
                                   int32_t n_segments, const DfcHyper* hypers, int32_t n_hypers,
                                   int32_t mode, const float* device_grad_scale,
                                   const int32_t* error_flag, const DfcCompressRange* next,
                                   uint32_t flags, int32_t ctas_per_sm, void* stream);

/*
 * The NVSwitch sum over every rank of numel bf16 values at a multicast
 * address, written as FP32 to out (device, 16-byte aligned): exactly the
 * gradient values the multicast form of dfc_zero_fused_step steps with.  No
 * reference counterpart; for checking the reduction.
 */
DFC_API int dfc_multicast_sum_bf16(const void* comp_multicast, float* out, int64_t numel,
                                   void* stream);

/*
 * Barrier across ranks on their streams.  slot_ptrs: host array of n_peers
 * device addresses of every rank's uint32 signal array (n_peers words each,
 * peer-mapped, zero before the first use).  Rank r stores `epoch` into word
 * r of every array (release, system scope), then waits until every word of
 * its own array has reached `epoch` (acquire, system scope), for at most
 * timeout_ns; on time-out it stores 1 + the index of the missing rank into
 * *error_flag (device int) and returns.  A flag that is already non-zero
 * (an earlier barrier gave up) makes the call return at once, storing
 * nothing into the peers' arrays and waiting for nothing, so a failed step
 * ends in bounded time on every rank.  Epochs must increase by one per call.
 * One rank per GPU: ranks sharing a GPU may never run concurrently.
 */
DFC_API int dfc_peer_barrier(uint32_t* const* slot_ptrs, int32_t n_peers, int32_t rank,
                             uint32_t epoch, int32_t* error_flag, int64_t timeout_ns,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DFC_B200_H_ */
