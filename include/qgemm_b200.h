/*
 * qgemm_b200.h -- C-ABI of the B200 (sm_100a) weight-only 4-bit GEMM path.
 *
 *   Y[M,N] = X[M,K] . W[N,K]^T      X bf16 row-major, W packed 4-bit along K,
 *                                    FP32 accumulation, Y bf16 (or fp32).
 *
 * The byte layouts are exactly those of titoatwork/qgemm-mx
 * include/qgemm/pack.hpp:14-85 (nibble 2i low / 2i+1 high, row-major linear
 * index n*K+k; scales in a separate array indexed n*(K/block)+k/block):
 *   MXFP4      E2M1 elements + one E8M0 byte per 32 along K
 *   NVFP4      E2M1 elements + one E4M3 byte per 16 along K + FP32 tensor scale
 *   INT4_G128  symmetric two's-complement nibbles + FP16 scale bits per 128
 *   INT4_G64   same, group 64
 * The reference exposes this path only as header-only C++ (no C-ABI); each
 * entry point below names the reference symbol whose behaviour it carries.
 *
 * Conventions
 *   - All data pointers are DEVICE pointers unless a parameter says otherwise;
 *     the caller owns every buffer.  Nothing here allocates device memory
 *     inside a GEMM call, synchronises, or reads back to the host, so every
 *     call is stream-ordered and can be captured into a CUDA graph (the
 *     reference's time_graphed protocol, timing.cuh:288-336).
 *   - `stream` is a cudaStream_t passed as void*.
 *   - Errors come back as qgemm_status_t; nothing throws or exits across the
 *     ABI.  Conditions on which the reference throws std::invalid_argument
 *     (pack.hpp:115,122,427-430,467,505-508) return QGEMM_ERR_INVALID_ARG.
 *     qgemm_last_error_message() gives the text for the calling thread.
 */
#ifndef QGEMM_B200_H
#define QGEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  QGEMM_OK = 0,
  QGEMM_ERR_INVALID_ARG = 1,      /* bad pointer/size/format (reference: throw) */
  QGEMM_ERR_UNSUPPORTED_SHAPE = 2,/* shape the kernels do not cover            */
  QGEMM_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed      */
  QGEMM_ERR_NCCL = 4,             /* an NCCL call failed                       */
  QGEMM_ERR_TIMEOUT = 5,          /* a bounded device-side wait gave up        */
  QGEMM_ERR_WORKSPACE = 6         /* workspace missing or too small            */
} qgemm_status_t;

/* Mirrors qgemm::Format (formats.cuh:16-24) for the 4-bit members; the dense
 * entries exist only for byte accounting. */
typedef enum {
  QGEMM_FMT_MXFP4 = 0,
  QGEMM_FMT_NVFP4 = 1,
  QGEMM_FMT_INT4_G128 = 2,
  QGEMM_FMT_INT4_G64 = 3,
  QGEMM_FMT_BF16 = 4,      /* accounting only */
  QGEMM_FMT_FP16 = 5,      /* accounting only */
  QGEMM_FMT_FP8_E4M3 = 6   /* accounting only */
} qgemm_format_t;

/* Layout of a packed matrix (qgemm_weights_t.layout).
 *   QGEMM_LAYOUT_CANONICAL      pack.hpp's bytes, as above.
 *   QGEMM_LAYOUT_SCALE_CHECKED  MXFP4 / NVFP4 only: the same bytes, which
 *       qgemm_repack has checked to hold no scale byte outside the range the
 *       decode kernel decodes by exponent arithmetic (MXFP4 E8M0 0x00 and
 *       0xFF; NVFP4 E4M3 zero, subnormal and NaN).  The TMA-fed decode
 *       kernel then skips its per-chunk search for such bytes; every other
 *       kernel reads the bytes as canonical.  Describing weights that hold
 *       such bytes with this layout gives unspecified values in the outputs
 *       their blocks reach. */
typedef enum { QGEMM_LAYOUT_CANONICAL = 0, QGEMM_LAYOUT_SCALE_CHECKED = 1 } qgemm_layout_t;

/* A packed weight matrix resident in device memory.  Replaces the reference's
 * PackedMxfp4 / PackedNvfp4 / PackedInt4 containers (pack.hpp:396-417), whose
 * std::vector members become device pointers of the same length and layout. */
typedef struct {
  int32_t format;          /* qgemm_format_t (4-bit members only)           */
  int32_t layout;          /* qgemm_layout_t (0 = the reference's bytes)     */
  size_t N, K;             /* W is [N, K]                                    */
  const uint8_t* data;     /* N*K/2 bytes                                    */
  const void* scales;      /* MXFP4/NVFP4: uint8 [N*K/blk]; INT4: uint16 bits */
  float tensor_scale;      /* NVFP4 per-tensor FP32 scale; ignored otherwise */
} qgemm_weights_t;

/* ---- library -------------------------------------------------------------- */
const char* qgemm_version(void);
const char* qgemm_status_string(qgemm_status_t s);
/* Message of the last failing call made by this host thread ("" if none). */
const char* qgemm_last_error_message(void);

/* ---- byte accounting: formats.cuh:40-109 ---------------------------------- */
double qgemm_bytes_per_weight(int32_t format);                   /* formats.cuh:67-69 */
size_t qgemm_weight_bytes(int32_t format, size_t N, size_t K);   /* formats.cuh:73-76 */
size_t qgemm_total_bytes(int32_t format, size_t M, size_t N, size_t K); /* :80-83 */
double qgemm_flops(size_t M, size_t N, size_t K);                /* formats.cuh:91-94 */
/* Exact buffer sizes of a packed matrix (pack.hpp:113-153). */
qgemm_status_t qgemm_packed_sizes(int32_t format, size_t N, size_t K,
                                  size_t* data_bytes, size_t* scale_bytes);

/* ---- packers: device quantize + pack, bit-exact to pack.hpp -------------- *
 * W is FP32 row-major [N,K] on the device.  Outputs use the reference layout.
 * Each returns QGEMM_ERR_INVALID_ARG on the reference's throw conditions.    */
/* pack.hpp:465-497 pack_mxfp4 */
qgemm_status_t qgemm_pack_mxfp4(const float* W, size_t N, size_t K,
                                uint8_t* data, uint8_t* scales, void* stream);
/* pack.hpp:502-542 pack_nvfp4 (tensor_scale: finite, > 0, host value) */
qgemm_status_t qgemm_pack_nvfp4(const float* W, size_t N, size_t K,
                                float tensor_scale, uint8_t* data,
                                uint8_t* scales, void* stream);
/* pack.hpp:424-462 pack_int4 (group 64 or 128; scales = FP16 bits) */
qgemm_status_t qgemm_pack_int4(const float* W, size_t N, size_t K, int32_t group,
                               uint8_t* data, uint16_t* scales, void* stream);
/* NVFP4 per-tensor scale max|W|/(448*6) into *out (device float).  The
 * reference takes this value as a caller argument (pack.hpp:502-508). */
qgemm_status_t qgemm_nvfp4_tensor_scale(const float* W, size_t n, float* out,
                                        void* stream);

/* ---- dequant: pack.hpp:548-585 dequant_{int4,mxfp4,nvfp4}, bit-exact ------ */
qgemm_status_t qgemm_dequant(const qgemm_weights_t* w, float* out, void* stream);

/* ---- scalar codecs on the device, bit-exact to pack.hpp:183-374 ----------- *
 * kind: 0 e2m1_encode -> uint8, 1 e8m0_encode -> uint8, 2 e4m3_encode -> uint8,
 *       3 float_to_fp16_bits -> uint16.                                      */
qgemm_status_t qgemm_codec_encode(int32_t kind, const float* in, void* out,
                                  size_t n, void* stream);

/* Code-level packers (pack.hpp:611-674): already-quantised codes into the
 * canonical layout, and back.  MXFP4 / NVFP4: codes are uint8 E2M1 codes
 * (the low 4 bits are packed, as pack_nibble masks them) and scales_in the
 * raw E8M0 / E4M3 scale bytes, copied unchanged (pack_mxfp4_codes,
 * pack_nvfp4_codes; an NVFP4 tensor scale is carried in qgemm_weights_t).
 * INT4: codes are int32 values clamped to [-8, 7] (int4_to_nibble) and
 * scales_in FP32 group scales, stored as FP16 bits (float_to_fp16_bits,
 * pack_int4_codes).  Unpacking returns the uint8 nibbles (unpack_e2m1_codes)
 * or the int32 signed values (unpack_int4_codes).  N*K must be even and K
 * divisible by the format's block, or QGEMM_ERR_INVALID_ARG, as the
 * reference throws (pack.hpp:113-139).  Device pointers, stream-ordered. */
qgemm_status_t qgemm_pack_codes(int32_t format, const void* codes, const void* scales_in,
                                size_t N, size_t K, uint8_t* data, void* scales, void* stream);
qgemm_status_t qgemm_unpack_codes(int32_t format, const uint8_t* data, size_t N, size_t K,
                                  void* codes, void* stream);

/* ---- layouts: the kernel-optimal layout as an offline transform ----------
 * The reference plans a kernel-optimal repacked layout derived from the
 * dequantisation sequence, with the canonical bytes as the parity format
 * (docs/D1_LAYOUT_DERIVATION.md:17-52).  Here it is
 * QGEMM_LAYOUT_SCALE_CHECKED (above).  qgemm_layout_sizes gives the buffer
 * sizes of a layout; qgemm_repack writes canonical weights (src->layout 0)
 * in `layout` (for the scale-checked layout it scans the scales, waits for
 * `stream`, and returns QGEMM_ERR_INVALID_ARG if a byte is outside the fast
 * range: such weights stay canonical); qgemm_unpack writes the canonical
 * bytes of weights in any layout.  The outputs may alias the source's
 * arrays (the bytes are then not copied).  Device pointers. */
qgemm_status_t qgemm_layout_sizes(int32_t format, int32_t layout, size_t N, size_t K,
                                  size_t* data_bytes, size_t* scale_bytes);
qgemm_status_t qgemm_repack(const qgemm_weights_t* src, int32_t layout, uint8_t* data,
                            void* scales, void* stream);
qgemm_status_t qgemm_unpack(const qgemm_weights_t* src, uint8_t* data, void* scales,
                            void* stream);

/* ---- GEMM ------------------------------------------------------------------
 * Workspace: scratch the kernels use for split-K partial sums, tile tickets
 * and the converted copy of X.  Size it with qgemm_workspace_size(); zero it
 * once before first use (qgemm_workspace_init or cudaMemsetAsync).  The
 * tickets sit at the start of every workspace in a region sized from N, and
 * every call returns them to zero, so one workspace of at least
 * qgemm_workspace_size(w, M) bytes for each M it meets (the size is not
 * monotone in M: the kernel changes) serves all those calls in stream order.
 * Calls that may overlap on the GPU need distinct workspaces.                */
size_t qgemm_workspace_size(const qgemm_weights_t* w, int32_t M);
qgemm_status_t qgemm_workspace_init(void* workspace, size_t ws_bytes, void* stream);
/* Number of kernel launches one qgemm_gemm_w4a16 call makes for (w, M), and
 * which GEMM kernel it uses (0 LDG-fed decode, 1 TMA-fed decode, 2 stream-K
 * tcgen05, 3 tile-per-CTA tcgen05, 4 block-scaled tcgen05 for MXFP4 with
 * 9 <= M <= 128).  Returns -1 for invalid arguments.  No
 * counterpart in the reference (its benches launch one kernel per GEMM);
 * used for launch accounting in benchmarks. */
int32_t qgemm_launch_count(const qgemm_weights_t* w, int32_t M, int32_t* kernel);

/* Y = X . W^T.  X: bf16 bits [M,K]; Y: bf16 bits [M,N].  Any M >= 1.
 * Result is within the reference GEMM (ref_gemm.hpp:15-27, double
 * accumulation) by max-abs <= 1e-2*||row||_inf and rel-Frobenius <= 1e-3. */
qgemm_status_t qgemm_gemm_w4a16(const qgemm_weights_t* w, const uint16_t* X,
                                int32_t M, uint16_t* Y, void* workspace,
                                size_t ws_bytes, void* stream);
/* Same, FP32 output (no final bf16 rounding). */
qgemm_status_t qgemm_gemm_w4a16_f32(const qgemm_weights_t* w, const uint16_t* X,
                                    int32_t M, float* Y, void* workspace,
                                    size_t ws_bytes, void* stream);

/* ---- grouped GEMM (mixture of experts) ------------------------------------
 * E weight sets w[0 .. E-1] of one format and shape (N, K).  Expert e
 * multiplies its M[e] activation rows, rows offs[e] .. offs[e] + M[e] - 1 of
 * X (bf16 bits [rows][K]), and writes the same rows of Y (bf16 bits
 * [rows][N]):  Y[offs[e] + i] = X[offs[e] + i] . W_e^T,  0 <= i < M[e].
 * M[e] = 0 skips expert e.  M and offs are host arrays: the routing counts
 * are on the host when the call is made.  The reference plans this as its
 * grouped / MoE variant with variable M per expert
 * (docs/PROJECT-v2.0-fp4-hopper.md:89-90, MASTER_EXECUTION_PLAN.md:249) and
 * does not build it; each expert's result is a qgemm_gemm_w4a16 result
 * (same bounds against ref_gemm.hpp:15-27).  Experts with 1 <= M[e] <= 16
 * (any format, K % 256 == 0) run up to 32 at a time as one X-preparation
 * launch and one decode-GEMM launch whose stream-K iteration space covers all
 * of them; other experts run as qgemm_gemm_w4a16 calls on the same stream.
 * workspace: qgemm_grouped_workspace_size(w, E, max_m) bytes serve every call
 * whose M[e] <= max_m; zero it once (qgemm_workspace_init).  A workspace
 * sized for both also serves qgemm_gemm_w4a16 calls. */
size_t qgemm_grouped_workspace_size(const qgemm_weights_t* w, int32_t E, int32_t max_m);
qgemm_status_t qgemm_grouped_gemm_w4a16(const qgemm_weights_t* w, int32_t E, const uint16_t* X,
                                        const int32_t* M, const int64_t* offs, uint16_t* Y,
                                        void* workspace, size_t ws_bytes, void* stream);

/* ---- tensor parallel over the GPUs of one node (W sharded along N) -------
 * No counterpart in the reference, which runs on one GPU; the sharding
 * (rank r holds rows [r N/world, (r+1) N/world) of W and its scales) and the
 * gather of Y are the multi-GPU step its bench is extended with.
 * qgemm_tp_gemm_w4a16 computes this rank's Y slice with qgemm_gemm_w4a16's
 * kernels, writes it into every rank's Y_full [M][N] through peer pointers
 * (y_peers[d] = rank d's Y_full as mapped in this process), adds its
 * arrival to every rank's sync block (system-scope release after the
 * stores) and waits (bounded, ~2 s) until every rank's arrival for this call
 * has reached its own sync block, i.e. all slices have landed in its own
 * Y_full.  Every rank makes the same
 * sequence of calls; a rank's Y_full is written by all ranks, so reuse a
 * buffer only once every rank is done reading the previous result.
 * sync_peers[d]: rank d's sync block, qgemm_tp_sync_bytes() bytes, zeroed
 * once.  workspace: qgemm_tp_workspace_size(w_local, M) bytes, zeroed once
 * (qgemm_workspace_init).  Graph-capturable: the arrival and expected
 * counts are device-side counters in the sync block. */
size_t qgemm_tp_sync_bytes(int32_t world);
size_t qgemm_tp_workspace_size(const qgemm_weights_t* w_local, int32_t M);
qgemm_status_t qgemm_tp_gemm_w4a16(const qgemm_weights_t* w_local, const uint16_t* X,
                                   int32_t M, int32_t world, int32_t rank,
                                   uint16_t* const* y_peers, uint32_t* const* sync_peers,
                                   void* workspace, size_t ws_bytes, void* stream);
/* QGEMM_ERR_TIMEOUT if a tp wait gave up (a peer never announced). */
qgemm_status_t qgemm_tp_status(int32_t* timed_out);
/* CUDA IPC: the 64-byte handle of the allocation holding dev_ptr and the
 * pointer's byte offset in it; mapping another process's allocation from
 * its handle (*dev_ptr = its base, add the offset) and unmapping it. */
qgemm_status_t qgemm_ipc_handle(const void* dev_ptr, uint8_t* handle64, size_t* offset);
qgemm_status_t qgemm_ipc_open(const uint8_t* handle64, void** dev_ptr);
qgemm_status_t qgemm_ipc_close(void* dev_ptr);

/* Y = X . W^T (bf16 out) without a workspace argument, for callers that
 * cannot provide one: an operator slot that passes only inputs, outputs and a
 * stream, a plugin inside a framework that owns the device memory pool and
 * forbids raw cudaMalloc, or code running while another component captures
 * the stream in global mode.  No counterpart in the reference (its host path
 * never needs device scratch).  Scratch is a fixed 16 MiB device array per
 * GPU held until exit; larger plans return QGEMM_ERR_WORKSPACE.  The first
 * call on a device looks up that array (make it before any stream capture);
 * every call shares it, so calls that may overlap on the GPU race.  Always
 * runs the decode kernel; allocates nothing. */
qgemm_status_t qgemm_gemm_w4a16_noalloc(const qgemm_weights_t* w, const uint16_t* X,
                                        int32_t M, uint16_t* Y, void* stream);

/* Synchronous: reports (and returns QGEMM_ERR_TIMEOUT) if a bounded barrier
 * wait inside a GEMM kernel gave up on this device; *faulted is then nonzero
 * and qgemm_last_error_message() names, per kernel family, where the first
 * wait gave up (warp, CTA and barrier index).  Not capturable. */
qgemm_status_t qgemm_umma_status(int32_t* faulted);

/* Synchronous: waits for the device, then resets every fault flag of the
 * current device (the GEMM kernels', the tensor-parallel exchange's and the
 * TMA probe's).  No counterpart in the reference, whose errors are fatal
 * (timing.cuh:36-44).  After a call that reported QGEMM_ERR_TIMEOUT its
 * outputs are wrong; the GEMM workspaces need nothing (every contributor of a
 * split tile takes its ticket even after a timeout, so the tickets return to
 * zero), but the tp sync blocks of every rank must be zeroed again
 * (qgemm_workspace_init) before the next tp call, since a rank that gave up
 * is a call ahead of its peers.  Then call this and continue.  Not
 * capturable. */
qgemm_status_t qgemm_clear_faults(void);

/* ---- baselines and probes (bench harness; not on the product path) ------- */
/* cuBLAS BF16 dense Y[M,N] = X[M,K] . W[N,K]^T (bench_cublas.cu:144-151 with
 * CUDA_R_16BF in place of CUDA_R_16F, COMPUTE_32F). */
qgemm_status_t qgemm_cublas_bf16_gemm(const uint16_t* W, const uint16_t* X,
                                      int32_t M, size_t N, size_t K, uint16_t* Y,
                                      void* stream);
/* cuBLASLt FP8 dense baseline, the one the reference plans for its "vs FP8"
 * headline (docs/BASELINE_STUDY.md:23, docs/MASTER_EXECUTION_PLAN.md:121,280;
 * no implementation there): W [N,K] and X [M,K] are E4M3 bytes, scale_w and
 * scale_x DEVICE pointers to their FP32 per-tensor scales, Y [M,N] bf16 =
 * (X.scale_x) . (W.scale_w)^T with FP32 accumulation.  K % 16 == 0,
 * N % 8 == 0, W, X, Y 16-byte aligned; workspace may be null (ws_bytes 0). */
qgemm_status_t qgemm_cublaslt_fp8_gemm(const uint8_t* W, const uint8_t* X,
                                       int32_t M, size_t N, size_t K,
                                       const float* scale_w, const float* scale_x,
                                       uint16_t* Y, void* workspace, size_t ws_bytes,
                                       void* stream);
/* Memory probes (bandwidth.cu:25-50, bench_stream_ideal.cu:29-39).
 * kind: 0 read-only with 128-bit loads, 1 read-only with TMA bulk copies
 * (cp.async.bulk, no multicast), 2 copy src->dst, 3 write-only fill dst.
 * bytes must be a multiple of 16; src/dst 16-byte aligned.                   */
qgemm_status_t qgemm_probe_launch(int32_t kind, const void* src, void* dst,
                                  size_t bytes, void* stream);
/* Synchronous: reports (and returns QGEMM_ERR_TIMEOUT) if a bounded wait in
 * a TMA bulk probe gave up on this device.  Not capturable. */
qgemm_status_t qgemm_probe_status(int32_t* timed_out);
/* SM count and L2 bytes of the current device (timing.cuh:50-91). */
qgemm_status_t qgemm_device_info(int32_t* sm_count, size_t* l2_bytes);

#ifdef __cplusplus
}
#endif
#endif /* QGEMM_B200_H */
