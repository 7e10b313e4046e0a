/*
 * mfcuda.h -- C ABI of the B200 (sm_100a) backend for manifesto's
 * data-parallel hot path: dtype conversion, packed Int4 group dequant,
 * axpy / scalar-broadcast vector loops, fused elementwise chains and
 * per-tensor amax-scaled FP8 quantisation (single tensor and whole
 * checkpoints sharded over several GPUs).
 *
 * Conventions
 *   - Plain C types only: pointers, int32_t/int64_t/size_t, float.
 *   - Every entry point returns an int status: MF_OK (0) or a negative
 *     MF_ERR_* code. Each negative code corresponds 1:1 to a sentinel in
 *     manifesto tensor/errors.go:10-72 (see the table beside the enum), so
 *     a cgo adapter maps them with a switch. The message of the most recent
 *     failure on the calling OS thread is available from mf_last_error().
 *   - Device pointers are plain CUDA device addresses on the device chosen
 *     with mf_init(). Stream and event handles are cudaStream_t / cudaEvent_t
 *     cast to void*; a NULL stream is the legacy default stream.
 *   - No entry point synchronises the host with the device except the ones
 *     whose name says so (mf_stream_sync, mf_event_sync, mf_device_sync) and
 *     the set-up calls (mf_init, mf_alloc, mf_free, mf_fused_compile,
 *     mf_comm_init). Scalar results such as amax are written to device
 *     memory, never returned to the host (manifesto
 *     scripts/check_banned.sh:28-40 forbids host syncs on the launch path).
 *   - Arithmetic follows manifesto's Go scalar code bit for bit, including
 *     its FP8 rounding quirks (compat = MF_COMPAT_REFERENCE). The file:line
 *     each entry point replaces is given in its comment; paths are inside
 *     the manifesto Go module.
 */
#ifndef MFCUDA_H
#define MFCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MFCUDA_ABI_VERSION 1

/* ---------------------------------------------------------------------
 * dtype wire codes: identical to dtype.DType (dtype/dtype.go:29-49).
 * ------------------------------------------------------------------- */
enum mf_dtype {
    MF_DT_INVALID = 0,
    MF_DT_F64 = 1,
    MF_DT_F32 = 2,
    MF_DT_F16 = 3,
    MF_DT_BF16 = 4,
    MF_DT_F8E4M3 = 5,
    MF_DT_F8E5M2 = 6,
    MF_DT_I64 = 7,
    MF_DT_I32 = 8,
    MF_DT_I16 = 9,
    MF_DT_I8 = 10,
    MF_DT_I4 = 11, /* packed two per byte, element 2i in the low nibble */
    MF_DT_U64 = 12,
    MF_DT_U32 = 13,
    MF_DT_U16 = 14,
    MF_DT_U8 = 15
};

/* ---------------------------------------------------------------------
 * Status codes.  Negative values map onto tensor/errors.go sentinels:
 *   MF_ERR_DTYPE_MISMATCH       -> tensor.ErrDTypeMismatch       (:13)
 *   MF_ERR_DTYPE_UNSUPPORTED    -> tensor.ErrDTypeUnsupported    (:18)
 *   MF_ERR_LAYOUT_UNSUPPORTED   -> tensor.ErrLayoutUnsupported   (:23)
 *   MF_ERR_SHAPE_MISMATCH       -> tensor.ErrShapeMismatch       (:28)
 *   MF_ERR_BACKEND_CLOSED       -> tensor.ErrBackendClosed       (:46)
 *   MF_ERR_SHAPE_INVALID        -> tensor.ErrShapeInvalid        (:50)
 *   MF_ERR_NEEDS_PLATFORM_SETUP -> tensor.ErrNeedsPlatformSetup  (:64)
 *   MF_ERR_ALLOCATOR_EXHAUSTED  -> tensor.ErrAllocatorExhausted  (:71)
 * The remaining codes have no sentinel and surface as wrapped errors.
 * ------------------------------------------------------------------- */
enum mf_status {
    MF_OK = 0,
    MF_ERR_INVALID_ARGUMENT = -1,
    MF_ERR_DTYPE_MISMATCH = -2,
    MF_ERR_DTYPE_UNSUPPORTED = -3,
    MF_ERR_LAYOUT_UNSUPPORTED = -4,
    MF_ERR_SHAPE_MISMATCH = -5,
    MF_ERR_BACKEND_CLOSED = -6,
    MF_ERR_SHAPE_INVALID = -7,
    MF_ERR_NEEDS_PLATFORM_SETUP = -8,
    MF_ERR_ALLOCATOR_EXHAUSTED = -9,
    MF_ERR_CUDA = -10,        /* a CUDA runtime call failed */
    MF_ERR_NCCL = -11,        /* an NCCL call failed */
    MF_ERR_DEVICE_STICKY = -12 /* a kernel recorded an error in device memory */
};

/* FP8 encoder semantics. REFERENCE reproduces dtype/fp8.go:77-136 and
 * :190-249 exactly (including the subnormal shift, the exponent-15
 * saturation of E4M3 and NaN -> 0x7f). OCP is the OCP FP8 rule with
 * saturation to the largest finite value (the sm_100 cvt .satfinite
 * result) and NaN -> 0x7f. */
enum mf_compat { MF_COMPAT_REFERENCE = 0, MF_COMPAT_OCP = 1 };

typedef void* mf_stream; /* cudaStream_t */
typedef void* mf_event;  /* cudaEvent_t */
typedef struct mf_fused_kernel_s* mf_fused_kernel;
typedef struct mf_comm_s* mf_comm;
typedef struct mf_ckpt_plan_s* mf_ckpt_plan;

/* ---------------------------------------------------------------------
 * Lifecycle and errors
 * ------------------------------------------------------------------- */
int mf_abi_version(void);
/* Number of CUDA devices; works without any device (returns 0). */
int mf_device_count(int* count);
/* Select and initialise `device` for all later calls of this process.
 * Replaces the device half of tensor.Backend construction
 * (tensor/backend.go:18-68). Idempotent. */
int mf_init(int device);
/* Release library-owned device resources. After it, kernels return
 * MF_ERR_BACKEND_CLOSED until mf_init is called again
 * (tensor.Backend.Close, tensor/backend.go:65-67). */
int mf_shutdown(void);
/* Message of the last failure on this OS thread ("" if none). The pointer
 * stays valid until the next failing call on the same thread. */
const char* mf_last_error(void);
/* Copy the last error message into buf (always NUL terminated). */
int mf_last_error_copy(char* buf, size_t n);
/* Read and clear the sticky device status (MF_OK or MF_ERR_DEVICE_STICKY
 * with a code in *device_code). Synchronises the device. Backs
 * tensor.Tensor.Sync (tensor/tensor.go:53-130). */
int mf_device_status(int* device_code);
/* Device status code of a bounded wait that gave up (a bulk-copy stage that
 * never landed, or mf_wait_flag's flag that was never set). */
#define MF_DEVICE_TIMEOUT 0x7100
/* Make `stream` wait until the int at device address `flag` equals `expect`
 * (acquire load, polled with a short sleep), for at most `max_polls` polls;
 * if it never does, record MF_DEVICE_TIMEOUT in the sticky status and let the
 * stream continue. The building block for a handshake with a peer rank or the
 * host that must not hang the GPU. No counterpart in the reference. */
int mf_wait_flag(const int* flag, int expect, int64_t max_polls, mf_stream stream);
/* Device properties used to size launches. */
int mf_device_info(int* sm_count, int* cc_major, int* cc_minor, size_t* total_bytes);

/* ---------------------------------------------------------------------
 * Memory, transfers, streams, events.  These back tensor.Backend.Upload /
 * UploadAsync / Download (tensor/backend.go:38-63) and the workspace
 * arena of runtime.WorkspaceAttacher.AttachWorkspace
 * (runtime/executor.go:42-48, sized by ir.WorkspaceLayout.Size,
 * ir/workspace.go:12-33).
 * ------------------------------------------------------------------- */
int mf_alloc(void** dptr, size_t bytes);           /* 256-byte aligned */
int mf_free(void* dptr);
int mf_host_alloc(void** hptr, size_t bytes);      /* page-locked host memory */
int mf_host_free(void* hptr);
int mf_memcpy_h2d_async(void* dst, const void* src, size_t bytes, mf_stream stream);
int mf_memcpy_d2h_async(void* dst, const void* src, size_t bytes, mf_stream stream);
int mf_memcpy_d2d_async(void* dst, const void* src, size_t bytes, mf_stream stream);
int mf_memset_async(void* dst, int value, size_t bytes, mf_stream stream);
/* Streams and events: ir.Node.StreamID and ir.SyncEvent
 * (ir/sync_event.go:14-26, ir/stream_scheduler.go:56-141) map onto these:
 * SyncEvent{Wait:false} -> mf_event_record, {Wait:true} -> mf_stream_wait_event. */
int mf_stream_create(mf_stream* stream);
int mf_stream_destroy(mf_stream stream);
int mf_stream_sync(mf_stream stream);
int mf_event_create(mf_event* event, int enable_timing);
int mf_event_destroy(mf_event event);
int mf_event_record(mf_event event, mf_stream stream);
int mf_stream_wait_event(mf_stream stream, mf_event event);
int mf_event_sync(mf_event event);
int mf_event_elapsed_ms(mf_event start, mf_event stop, float* ms);
int mf_device_sync(void);

/* ---------------------------------------------------------------------
 * K1-K3: dtype conversion.
 * Replaces the element loops of convert.BytesToFloat32 / BytesToBFloat16 /
 * BytesToFloat16 / BytesToFloat8E4M3 / BytesToFloat8E5M2
 * (dtype/convert/convert.go:85-228) and the store encoders
 * float32VectorBytes (runtime/axpy.go:171-194) and Float32AsDTypeBytes
 * (runtime/session.go:431-452).  Every conversion decodes src to float32
 * exactly as BytesToFloat32 does, then encodes with the scalar encoder of
 * dst_dtype (NewBfloat16FromFloat32 bfloat16.go:41-55, Fromfloat32
 * float16.go:109-111, NewF8E4M3FromFloat32 fp8.go:77-136,
 * NewF8E5M2FromFloat32 fp8.go:190-249).
 * src dtypes: F64 F32 F16 BF16 F8E4M3 F8E5M2 I64 I32 I16 I8 I4 U64 U32 U16 U8.
 * dst dtypes: F32 F16 BF16 F8E4M3 F8E5M2.
 * n counts logical elements; for I4 the source holds (n+1)/2 bytes.
 * ------------------------------------------------------------------- */
int mf_convert(int src_dtype, int dst_dtype, const void* src, void* dst,
               int64_t n, int compat, mf_stream stream);

/* ---------------------------------------------------------------------
 * K4: packed Int4 group dequantisation (config: 4096x14336, group 128).
 *   out[r, c] = encode_out( float32(q[r, c]) * float32(scales[r, c / group]) )
 * q is row-major [rows, cols] packed two nibbles per byte, element 2i in
 * the low nibble, sign-extended (dtype/int4.go:60-78,
 * dtype/convert/decoders.go:262-289); cols must be even so rows start on
 * byte boundaries.  scales is row-major [rows, ceil(cols/group)] of
 * scale_dtype (BF16, F16 or F32).  out_dtype is BF16 (NewBfloat16FromFloat32
 * rounding), F16 or F32.  The group scale itself has no counterpart in the
 * reference, which only sign-extends nibbles.
 * ------------------------------------------------------------------- */
int mf_int4_dequant_grouped(const void* q, const void* scales, int scale_dtype,
                            void* out, int out_dtype, int64_t rows, int64_t cols,
                            int64_t group, mf_stream stream);

/* ---------------------------------------------------------------------
 * K5: y <- y + alpha * x, in place on y.
 * Replaces axpyDevice.Axpy(y, x, count, alpha, format)
 * (runtime/axpy.go:13-15, called at :84-90) and the host loops of
 * axpyOntoHost (:115-117 for F32, :145-147 + :171-194 for BF16/F16).
 * Arithmetic: float32 multiply then float32 add, two roundings, no FMA
 * (the amd64 Go build does not contract).  fused_fma = 1 selects a single
 * rounding, which is what an arm64 Go build produces.
 * dtype: F32, BF16 or F16 (BF16/F16 decode to float32, compute, re-encode).
 * ------------------------------------------------------------------- */
int mf_axpy(void* y, const void* x, int64_t n, float alpha, int dtype,
            int fused_fma, mf_stream stream);

/* K6: out[i] = src[i] (op) scalar in float32, then encoded to dst_dtype.
 * Replaces applyScalarBroadcast (runtime/executor_math.go:195-234) and
 * its store encode (writeFloat32VectorOutput, :254-292).
 * op: 0 add, 1 sub, 2 mul, 3 div (div by 0 is rejected like :222-224). */
enum mf_scalar_op { MF_SCALAR_ADD = 0, MF_SCALAR_SUB = 1, MF_SCALAR_MUL = 2, MF_SCALAR_DIV = 3 };
int mf_scalar_broadcast(const void* src, int src_dtype, void* dst, int dst_dtype,
                        int64_t n, float scalar, int op, mf_stream stream);
/* math.linspace (runtime/executor_math.go:57-108) written straight into device
 * memory as F32, BF16 or F16 (the store encode of writeLinspaceOutput):
 * v[i] = start + float32(i) * ((stop - start) / float32(intervals)), intervals =
 * count - 1 (count when endpoint is 0), v[0] = start and v[count-1] = stop when the
 * endpoint is included. count <= 0 is MF_ERR_INVALID_ARGUMENT ("count must be
 * positive"). */
int mf_linspace(float start, float stop, int64_t count, int endpoint, void* dst, int dst_dtype,
                mf_stream stream);

/* ---------------------------------------------------------------------
 * K7: fused elementwise chains (optimizer.FusionAST, optimizer/fusion_ast.go:86-113).
 * The program is the FusionAST in postfix order: op[i] is an
 * optimizer.NodeType value (optimizer/fusion_ast.go:32-65: 1 Input,
 * 2 Constant, 3 Add, 4 Sub, 5 Mul, 6 Div, 7 Max, 8 Min, 9 Neg, 10 Abs,
 * 11 Sqrt, 12 Exp, 13 Log, 14 ReLU, 15 Sigmoid, 16 Tanh, 17 Silu,
 * 18 Gelu, 19 LeakyReLU); arg[i] is the input index for Input and the
 * index into consts for Constant, unused otherwise.
 * Per element the kernel decodes every input to float32, evaluates the
 * tree with codegen/cpu.go:126-212 semantics (binary ops and
 * Neg/Abs/ReLU/LeakyReLU in float32; Sqrt/Exp/Log/Sigmoid/Tanh/Silu/Gelu
 * in float64 rounded to float32) and encodes the result to out_dtype.
 * in_bcast[j] = 0 means input j has n elements; L > 0 means input j has L
 * elements and is read at index (i mod L) (broadcast over the last
 * dimension; the reference requires full-size inputs, cpu.go:78-85).
 * Replaces CPUKernel.Run (codegen/cpu.go:59-92).
 * ------------------------------------------------------------------- */
#define MF_FUSED_MAX_NODES 64
#define MF_FUSED_MAX_INPUTS 8
#define MF_FUSED_MAX_CONSTS 32
typedef struct mf_fused_program {
    int32_t n_nodes;
    const int32_t* op;
    const int32_t* arg;
    int32_t n_consts;
    const double* consts;
    int32_t n_inputs;
    const int32_t* in_dtype;  /* F32, F16 or BF16 */
    const int64_t* in_bcast;  /* see above; NULL = all full-size */
    int32_t out_dtype;        /* F32, F16 or BF16 */
} mf_fused_program;

/* Validate a program; picks a hand-specialised kernel when the program
 * matches one (e.g. Mul(Silu(Add(Mul(x,g),b)),y)), and emits CUDA source for
 * the expression and compiles it with NVRTC for sm_100a (the CUDA
 * counterpart of the Metal target's shader emission, codegen/metal.go:79-227;
 * 0.1-0.5 s, once per distinct program in a process).  The generated code
 * has three kernels: a bulk-copy pipeline over whole tiles of the full-size
 * inputs (16-byte aligned buffers, broadcast lengths that are multiples of 8,
 * at least one tile per SM), an 8-elements-per-lane kernel for smaller aligned
 * arrays, and an element-wise one for everything else.  MF_FUSED_JIT_DUMP=dir
 * writes each generated source to dir (a debugging aid).  Without NVRTC the
 * runtime interpreter runs the program.  Needs no device. */
int mf_fused_compile(const mf_fused_program* program, mf_fused_kernel* kernel);
int mf_fused_destroy(mf_fused_kernel kernel);
/* Which device code runs the kernel: 1 a hand-specialised body (the SwiGLU
 * chain; when its generated code's bulk-copy pipeline applies to a launch --
 * aligned buffers, at least one tile per SM -- that pipeline runs instead,
 * measured faster with the same codes), 2 CUDA source generated for this
 * expression and compiled with NVRTC for sm_100a at mf_fused_compile, 0 the
 * runtime interpreter (used when NVRTC is unavailable or MF_FUSED_JIT=0;
 * mf_last_error then gives the reason). */
int mf_fused_is_specialised(mf_fused_kernel kernel, int* specialised);
/* out: n elements of out_dtype.  If d_amax is not NULL, the kernel also
 * folds max|out| (of the encoded values, NaN ignored) into *d_amax with an
 * atomic max; *d_amax must be initialised (e.g. to 0) by the caller. */
int mf_fused_launch(mf_fused_kernel kernel, const void* const* inputs, void* out,
                    int64_t n, float* d_amax, mf_stream stream);

/* ---------------------------------------------------------------------
 * K8: per-tensor amax-scaled FP8 quantisation.  No counterpart in the
 * reference (which has no amax or scale op); built from its primitives:
 *   amax      = max |v| over the tensor (NaN ignored, Go '>' semantics)
 *   scale     = fp8_max / amax in float32 (fp8_max 448 for E4M3, 57344 for E5M2);
 *               scale = 1 when amax == 0 or amax is not finite
 *   q[i]      = encode_fp8(v[i] * scale)   (float32 multiply, compat rules)
 *   scale_inv = 1 / scale in float32 (stored for dequantisation)
 * ------------------------------------------------------------------- */
/* Fold max|src| into *d_amax (atomic max; caller initialises *d_amax). */
int mf_amax(const void* src, int src_dtype, int64_t n, float* d_amax, mf_stream stream);
/* Cast with the scale derived from *d_amax; writes *d_scale_inv if not NULL. */
int mf_fp8_scaled_cast(const void* src, int src_dtype, void* dst, int fp8_dtype,
                       const float* d_amax, float* d_scale_inv, int64_t n,
                       int compat, mf_stream stream);
/* amax + cast in one call.  d_amax is a caller-provided device float used
 * as scratch (and left holding the amax). */
int mf_fp8_quantize(const void* src, int src_dtype, void* dst, int fp8_dtype,
                    float* d_amax, float* d_scale_inv, int64_t n, int compat,
                    mf_stream stream);
/* Fused chain -> pre-cast store -> amax -> scaled FP8 in two passes:
 * pass 1 runs the fused program, writes `precast` (n values of the
 * program's out_dtype) and folds amax; pass 2 casts precast to FP8. */
int mf_fused_fp8(mf_fused_kernel kernel, const void* const* inputs, void* precast,
                 void* dst, int fp8_dtype, float* d_amax, float* d_scale_inv,
                 int64_t n, int compat, mf_stream stream);

/* ---------------------------------------------------------------------
 * K9: whole-checkpoint FP8 quantisation, tensors row-split over ranks.
 * ------------------------------------------------------------------- */
/* One contiguous chunk of one tensor owned by this rank. */
typedef struct mf_chunk_desc {
    const void* src;   /* n elements of src_dtype (F32, F16 or BF16) */
    void* dst;         /* n FP8 bytes */
    int64_t n;
    int32_t tensor;    /* index into the amax / scale_inv vectors */
    int32_t src_dtype;
} mf_chunk_desc;

/* Row split: tensor t of rows[t] x cols[t] elements is cut into `world`
 * contiguous row ranges whose sizes differ by at most one row; rank r owns
 * range r.  Writes first_row[t] and n_rows[t] for `rank`.  Host only. */
int mf_ckpt_partition(const int64_t* rows, int32_t n_tensors, int32_t world,
                      int32_t rank, int64_t* first_row, int64_t* n_rows);

/* NCCL communicator for the amax exchange.  mf_comm_unique_id writes 128
 * bytes (ncclUniqueId) on rank 0; the host sends them to every rank by any
 * means (torch.distributed store, MPI, a file); each rank then calls
 * mf_comm_init with its rank. */
int mf_comm_unique_id(void* id128);
int mf_comm_init(mf_comm* comm, int32_t world, int32_t rank, const void* id128);
int mf_comm_destroy(mf_comm comm);
/* In-place max all-reduce of a float vector in device memory. */
int mf_comm_allreduce_max_f32(mf_comm comm, float* d_vec, int64_t count, mf_stream stream);

/* The two passes on their own, for callers that run the amax exchange with
 * their own collective: pass 1 folds max|chunk| into d_amax[chunk.tensor]
 * (atomic max; the caller zeroes d_amax first); pass 2 casts every chunk
 * with the scale of d_amax[chunk.tensor] and writes d_scale_inv (if not
 * NULL).  One grouped launch per 512 chunks each. */
int mf_ckpt_amax_pass(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                      float* d_amax, mf_stream stream);
int mf_ckpt_cast_pass(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                      const float* d_amax, float* d_scale_inv, int fp8_dtype, int compat,
                      mf_stream stream);

/* Quantise every chunk: pass 1 folds per-tensor amax of this rank's
 * chunks into d_amax[n_tensors] (zeroed by this call), then, if comm is
 * not NULL, an NCCL max all-reduce makes d_amax global, then pass 2 casts
 * every chunk with its tensor's scale and writes d_scale_inv[n_tensors].
 * Two grouped kernel launches and at most one collective; no host sync. */
int mf_ckpt_quant_fp8(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                      float* d_amax, float* d_scale_inv, int fp8_dtype, int compat,
                      mf_comm comm, mf_stream stream);

/* No counterpart in the reference.  The same quantisation as
 * mf_ckpt_quant_fp8 for callers that cannot provide device memory for the
 * per-tensor amax vector -- for example a host whose device memory all
 * belongs to another allocator, such as an executor that only holds the
 * workspace arena its graph planner sized in advance, or a deployment that
 * forbids cudaMalloc after set-up.  The amax vector lives in a static device
 * array inside the library instead (at most 4096 tensors, 16 KB per GPU,
 * held until the process exits); larger n_tensors return
 * MF_ERR_ALLOCATOR_EXHAUSTED.  Nothing is allocated.  Every call on a device
 * shares that array, so calls that overlap on the GPU race; each call zeroes
 * the entries it uses.  Every call looks the array's device address up with
 * the library's device current (nothing is cached, so a context the host
 * tears down and creates again is safe); the first call on a device also
 * loads the array there, so make it before any stream capture. */
int mf_ckpt_quant_fp8_noalloc(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                              float* d_scale_inv, int fp8_dtype, int compat, mf_comm comm,
                              mf_stream stream);

/* ---------------------------------------------------------------------
 * The checkpoint quantisation step in one launch.  Replaces the same Go
 * callers as mf_ckpt_quant_fp8 (the reference itself has no quantiser; the
 * per-tensor rule is the one of mf_fp8_quantize, the encoder
 * NewF8E4M3FromFloat32 dtype/fp8.go:77-136 / NewF8E5M2FromFloat32
 * :190-249).  Same codes, scale_inv and amax as mf_ckpt_quant_fp8 with the
 * same chunk table, bit for bit.
 *
 * A plan is built once per chunk table (like the workspace plan of
 * ir.PlanWorkspace, ir/planner.go:43-96): the tensors are cut into groups of
 * consecutive tensors of at most group_bytes of this rank's source (0 = 32 MB;
 * tensor_numel, the global element count of every tensor, makes every rank cut
 * the same groups; required when world > 1, NULL = this rank's counts), the chunk table and
 * group table go to device memory, and a small exchange buffer is allocated.
 * One run is one cooperative kernel: per group an amax phase, then (one group
 * later, the group's source still in L2) a cast phase, with the per-group amax
 * exchanged between the ranks inside the kernel through the ranks' exchange
 * buffers (CUDA IPC peer memory, plain stores and system-scope flags; every
 * wait bounded, a wait that runs out leaves MF_DEVICE_TIMEOUT in the sticky
 * status).  All chunks of a plan share one source dtype (F32, F16 or BF16).
 *
 * world > 1: create on every rank, pass each rank's 64-byte ipc_handle to all
 * ranks (in rank order, world * 64 bytes) to mf_ckpt_plan_connect, and make
 * sure every rank has connected before any rank runs (a barrier).  Every rank
 * must run the plan the same number of times.  A plan is not shared between
 * streams that run at once.  Destroy on every rank after every rank's last
 * run has finished (a barrier). */
int mf_ckpt_plan_create(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                        const int64_t* tensor_numel, int64_t group_bytes, int32_t world, int32_t rank,
                        int fp8_dtype, int compat, mf_ckpt_plan* plan, void* ipc_handle);
int mf_ckpt_plan_connect(mf_ckpt_plan plan, const void* ipc_handles);
/* One step: d_amax[n_tensors] (may be NULL) gets the global amax,
 * d_scale_inv[n_tensors] (may be NULL) amax / fp8_max, the chunks' dst the
 * codes.  One kernel launch; no host sync. */
int mf_ckpt_plan_run(mf_ckpt_plan plan, float* d_amax, float* d_scale_inv, mf_stream stream);
/* The same step in two launches, with the exchange fused into them instead of
 * a collective between them (same codes, amax and scale_inv, bit for bit):
 *   passes & 1  the amax pass: every source byte read once, this rank's
 *               per-tensor maxima folded into the plan's scratch; when world > 1
 *               the launch's last CTA stores them into this rank's slot of
 *               every rank's exchange buffer and sets its flag there (no
 *               collective call, no memset: the scratch of a run is cleared by
 *               the run before);
 *   passes & 2  the cast pass: its CTAs start streaming their tiles at once,
 *               wait (bounded) for every rank's flag of the run, take the
 *               maximum over the slots and cast; its CTA 0 writes d_amax and
 *               d_scale_inv (either may be NULL).
 * passes = 3 runs both; 1 then 2 (the bench times them apart) is the same.  A
 * run's amax pass must be followed by its cast pass before the next run, in
 * either form (MF_ERR_INVALID_ARGUMENT otherwise).  Two launches, no host sync. */
int mf_ckpt_plan_run_passes(mf_ckpt_plan plan, int passes, float* d_amax, float* d_scale_inv, mf_stream stream);
int mf_ckpt_plan_info(mf_ckpt_plan plan, int32_t* n_groups, int32_t* grid, int64_t* elements);
int mf_ckpt_plan_destroy(mf_ckpt_plan plan);

/* ---------------------------------------------------------------------
 * Measurement.  No counterpart in the reference (it has no device code).
 * mf_bw_probe moves bytes in a fixed read:write mix with the bulk-copy engine
 * alone (32 KB cp.async.bulk loads into shared memory and stores out of it,
 * no thread touches the data); its rate is the DRAM ceiling of that mix, the
 * denominator for a kernel with the same mix.  One step reads in_per_step
 * 16-byte vectors (read k of step s at src + 16 * (k * n_steps + s)) and
 * writes out_per_step (same layout in dst).  Mixes: (1,0) read-only,
 * (0,1) write-only, (1,1) copy, (1,4) decode-shaped, (2,1) cast-shaped.
 * Buffers 16-byte aligned. */
int mf_bw_probe(const void* src, int in_per_step, void* dst, int out_per_step, int64_t n_steps,
                mf_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* MFCUDA_H */
