/*
 * cim22_cuda.h - C ABI of the B200 (sm_100a) execution backend for the
 * software-simulated CIM22 path.
 *
 * Plain C types only: pointers, sizes, status integers and caller-owned error
 * buffers. No exceptions cross this boundary. Every entry point that can fail
 * returns 0 on success and nonzero on failure; when an error buffer is given,
 * the diagnostic is copied into it NUL-terminated and truncated to the
 * capacity, the same convention as the reference's copyError
 * (runtime/Runtime.cpp:64-71).
 *
 * Three levels are exposed:
 *   1. The transaction executor, a drop-in for the reference's CIMRunner
 *      interface (include/CIM22/Execution/CIMRunner.h:75-154).
 *   2. The tile dispatch ABI that compiled model libraries call
 *      (_mlir_ciface_cim22_dispatch*, runtime/include/Session.h:52-66), routed
 *      to a CUDA session instead of the software runner.
 *   3. Layer-level entry points over device memory, which run whole CIM layers
 *      (every column, every 16-lane N tile and 64-element K tile) in a few
 *      launches. These replace the compiler-emitted Host glue around the
 *      tile calls (lib/Conversion/LinalgToCIM/Passes.cpp:760-857,2304-2476).
 */
#ifndef CIM22_CUDA_H
#define CIM22_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CIM22_CUDA_ABI_VERSION 1

/* Crossbar geometry of target profile cim22-4x5-v1
 * (include/CIM22/Execution/CIMRunner.h:19-22). */
#define CIM22_TILE_K 64
#define CIM22_TILE_N 16
#define CIM22_CACHE_ROWS 8
#define CIM22_MACRO_SLOTS 40

/* ------------------------------------------------------------------------ */
/* Transaction description. Field-for-field the data of
 * cim22::execution::CIMTransaction (include/CIM22/Execution/CIMExecutable.h:21-148);
 * the board-only `resource` string and flit stream are not needed to execute. */

typedef enum cim22_data_type {
  CIM22_DATA_INT8 = 0,
  CIM22_DATA_BF16 = 1
} cim22_data_type;

/* Same order as CIMPacketKind (CIMExecutable.h:25-33). */
typedef enum cim22_packet_kind {
  CIM22_PACKET_CONTROL = 0,
  CIM22_PACKET_WEIGHT = 1,
  CIM22_PACKET_WEIGHT_EXPONENT = 2,
  CIM22_PACKET_WORK = 3,
  CIM22_PACKET_INPUT_CACHE_WRITE = 4,
  CIM22_PACKET_RETURN_ROUTE = 5,
  CIM22_PACKET_OUTPUT_CACHE_READ = 6
} cim22_packet_kind;

/* Same order as BF16Compensation (include/CIM22/Execution/BF16Compensation.h:8). */
typedef enum cim22_bf16_compensation {
  CIM22_BF16_NONE = 0,
  CIM22_BF16_LEGACY = 1,
  CIM22_BF16_SIGN_SPLIT = 2
} cim22_bf16_compensation;

typedef struct cim22_frame_packet {
  int32_t kind; /* cim22_packet_kind */
  int32_t route[6];
  int64_t group_id;
  int64_t work_id;
  int64_t macro_slot;
  int64_t cache_address;
  int32_t test_core[3];
  int32_t data_type; /* cim22_data_type */
} cim22_frame_packet;

/* StaticWeightSection: values is lane-major [16][64]; exponents holds one
 * prealigned exponent per output lane (BF16 only). words are the board words,
 * compared for weight identity only. */
typedef struct cim22_static_weight {
  int64_t group_id;
  int64_t work_id;
  int64_t core_slot;
  int64_t macro_slot;
  int32_t route[6];
  const int32_t *words;
  int64_t num_words;
  int8_t values[16 * 64];
  uint8_t exponents[16];
  int32_t data_type;
} cim22_static_weight;

typedef struct cim22_input_binding {
  int64_t group_id;
  int64_t work_id;
  int64_t macro_slot;
  int64_t input_slot;
  int32_t data_type;
  int64_t input_cache_address;
} cim22_input_binding;

typedef struct cim22_readback_binding {
  int64_t group_id;
  int64_t work_id;
  int64_t macro_slot;
  int64_t output_cache_address;
  int32_t route[6];
  int32_t test_core[3];
  int32_t data_type;
} cim22_readback_binding;

typedef struct cim22_work {
  int64_t work_id;
  int64_t core_slot;
  int64_t macro_slot;
  int32_t route[6];
} cim22_work;

typedef struct cim22_group {
  int64_t group_id;
  const cim22_work *works;
  int64_t num_works;
} cim22_group;

typedef struct cim22_transaction {
  const char *target_profile;
  int64_t target_profile_version;
  int64_t execution_plan_version;
  const cim22_group *groups;
  int64_t num_groups;
  const cim22_static_weight *weights;
  int64_t num_weights;
  const cim22_frame_packet *packets;
  int64_t num_packets;
  const cim22_input_binding *inputs;
  int64_t num_inputs;
  const cim22_readback_binding *readbacks;
  int64_t num_readbacks;
} cim22_transaction;

/* Trace events, same kinds and fields as CIMTraceEvent (CIMRunner.h:46-73). */
typedef enum cim22_trace_kind {
  CIM22_TRACE_BEGIN_RUN = 0,
  CIM22_TRACE_CONFIGURE_WEIGHT = 1,
  CIM22_TRACE_CONFIGURE_INPUT = 2,
  CIM22_TRACE_SELECT_MACRO = 3,
  CIM22_TRACE_START_WORK = 4,
  CIM22_TRACE_CONFIGURE_RETURN_ROUTE = 5,
  CIM22_TRACE_READ_OUTPUT = 6,
  CIM22_TRACE_COMPLETE = 7,
  CIM22_TRACE_ERROR = 8
} cim22_trace_kind;

typedef struct cim22_trace_event {
  uint64_t sequence;
  int32_t kind;
  int64_t group_id;
  int64_t work_id;
  int64_t macro_slot;
  int64_t packet_index;
  int64_t cache_row_or_address;
} cim22_trace_event;

typedef void (*cim22_trace_callback)(void *context,
                                     const cim22_trace_event *event);

/* ------------------------------------------------------------------------ */
/* 1. Transaction executor (replaces CIMSoftwareRunner behind CIMRunner,
 *    include/CIM22/Execution/CIMRunner.h:75-154, lib/Execution/CIMSoftwareRunner.cpp). */

typedef struct cim22_cuda_runner cim22_cuda_runner;
typedef struct cim22_cuda_plan cim22_cuda_plan;

/* Executor context on one CUDA device. It owns the weight catalog (exact
 * payload interning, WeightResidency.h:28-50), the 40-slot residency table
 * with its write/hit counters (WeightResidency.h:59-92) and the device copies
 * of every interned weight tile. Calls on one runner must be serialized by the
 * caller, as a Session serializes its runner (runtime/Runtime.cpp:297). */
cim22_cuda_runner *cim22_cuda_runner_create(int device, char *error,
                                            size_t error_capacity);
void cim22_cuda_runner_destroy(cim22_cuda_runner *runner);

/* Resolve bindings, waves and readback packets once
 * (CIMSoftwareRunner::Plan, CIMSoftwareRunner.cpp:211-287) and upload the
 * transaction's weight tiles. The transaction is copied; the caller may free
 * it afterwards. batch_readbacks selects the batched-wave plan used by the
 * session dispatch (runtime/Runtime.cpp:204). */
cim22_cuda_plan *cim22_cuda_plan_create(cim22_cuda_runner *runner,
                                        const cim22_transaction *transaction,
                                        int batch_readbacks, char *error,
                                        size_t error_capacity);
void cim22_cuda_plan_destroy(cim22_cuda_plan *plan);

/* Execute one transaction synchronously (CIMSoftwareRunner::run,
 * CIMSoftwareRunner.cpp:289-482). inputs[i] is a host row of 64 int8 or 64
 * raw BF16 (uint16) values in dynamic-input binding order; outputs[i] is a
 * host row of 16 int32 or 16 uint16 values in readback binding order. Rows may
 * alias one another; a row read after an earlier wave published into the same
 * bytes sees the published values, as on the CPU. With use_residency, weights
 * are matched per physical slot and the slots are cleared on failure
 * (CIMRunner.h:133-145). Returns 0 or 1; outputs may be partially written on
 * failure (CIMRunner.h:79-80). */
int cim22_cuda_runner_run(cim22_cuda_runner *runner,
                          const cim22_cuda_plan *plan,
                          int32_t bf16_compensation, const void *const *inputs,
                          int64_t num_inputs, void *const *outputs,
                          int64_t num_outputs, int use_residency,
                          cim22_trace_callback trace, void *trace_context,
                          char *error, size_t error_capacity);

/* Residency counters (CIMWeightStats, WeightResidency.h:52-57). */
void cim22_cuda_runner_weight_stats(const cim22_cuda_runner *runner,
                                    uint64_t *writes, uint64_t *hits);
void cim22_cuda_runner_clear_residency(cim22_cuda_runner *runner);

/* ------------------------------------------------------------------------ */
/* 2. Session and the tile dispatch ABI of compiled model libraries.
 *
 * A CUDA session holds the model's transactions in id order (what
 * cim22_session_load_shared decodes from the model artifact,
 * runtime/Runtime.cpp:73-114) and executes them on one runner. Binding it to
 * the calling thread routes the four _mlir_ciface_cim22_dispatch* symbols to
 * it, as cim22_session_invoke binds activeSession (runtime/Runtime.cpp:333-336). */

typedef struct cim22_cuda_session cim22_cuda_session;

cim22_cuda_session *cim22_cuda_session_create(int device, char *error,
                                              size_t error_capacity);
void cim22_cuda_session_destroy(cim22_cuda_session *session);
/* Appends a transaction; its id is the previous transaction count. kernel_name
 * prefixes runner errors as "kernel: message" (runtime/Runtime.cpp:215-217). */
int64_t cim22_cuda_session_add_transaction(cim22_cuda_session *session,
                                           const cim22_transaction *transaction,
                                           const char *kernel_name, char *error,
                                           size_t error_capacity);
int64_t cim22_cuda_session_num_transactions(const cim22_cuda_session *session);
/* Starts an invocation on the calling thread: clears the error and the
 * dispatch counter and makes the session the target of the dispatch symbols.
 * end_invoke unbinds it, clears residency after an error
 * (runtime/Runtime.cpp:337-338) and returns 0 when no dispatch failed. */
void cim22_cuda_session_begin_invoke(cim22_cuda_session *session);
int cim22_cuda_session_end_invoke(cim22_cuda_session *session);
uint64_t cim22_cuda_session_dispatch_count(const cim22_cuda_session *session);
/* Borrowed; valid until the next call on the session. */
const char *cim22_cuda_session_error(const cim22_cuda_session *session);

/* MLIR ranked memref descriptor of rank 2 (StridedMemRefType<T, 2>). */
typedef struct cim22_memref2d {
  void *allocated;
  void *aligned;
  int64_t offset;
  int64_t sizes[2];
  int64_t strides[2];
} cim22_memref2d;

/* Generated model code calls these with [R,64] input and [R,16] output
 * memrefs (runtime/Runtime.cpp:221-247). Errors land in the bound session. */
void _mlir_ciface_cim22_dispatch(int64_t id, cim22_memref2d *input,
                                 cim22_memref2d *output);
void _mlir_ciface_cim22_dispatch_sign_split(int64_t id, cim22_memref2d *input,
                                            cim22_memref2d *output);
void _mlir_ciface_cim22_dispatch_legacy(int64_t id, cim22_memref2d *input,
                                        cim22_memref2d *output);
void _mlir_ciface_cim22_dispatch_int8(int64_t id, cim22_memref2d *input,
                                      cim22_memref2d *output);

/* ------------------------------------------------------------------------ */
/* 2b. Compiled model libraries on a CUDA session.
 *
 * A model library exports `const CIM22ModelV1 *cim22_model_v1(void)`
 * (include/CIM22/Runtime/ModelABI.h): ABI version 1, the Protobuf model
 * artifact (schema/cim22_model.proto) and the MLIR packed-argument entry
 * point. These functions replace cim22_session_* of runtime/Runtime.cpp
 * with the same arguments, return values and error texts; the artifact's
 * transactions run on a CUDA session instead of the software runner. */

typedef struct cim22_cuda_model cim22_cuda_model;

/* Decode and check an artifact (runtime/src/ModelArtifact.cpp:101-266,
 * 444-478) without loading anything. Returns 0 when it is valid, else 1 with
 * "invalid CIM22 Protobuf model: <reason>; recompile the model". */
int cim22_cuda_model_validate(const uint8_t *data, uint64_t size, char *error,
                              size_t error_capacity);
/* Replaces cim22_session_load_shared (runtime/Runtime.cpp:73-114): dlopen
 * (RTLD_NOW | RTLD_LOCAL), cim22_model_v1 ABI check ("incompatible CIM22
 * model ABI"), artifact decode and check, then every kernel's transaction
 * planned on a CUDA session on `device`. This library is promoted to global
 * symbol scope first, so the model's _mlir_ciface_cim22_dispatch* references
 * resolve to the CUDA dispatch above. */
cim22_cuda_model *cim22_cuda_model_load_shared(const char *path, int device, char *error,
                                               size_t error_capacity);
void cim22_cuda_model_destroy(cim22_cuda_model *model);
/* runtime/Runtime.cpp:252-291: -1 (or 0 for the count, "null session" for the
 * error) on a null model or an index out of range. dtype is the artifact's
 * DataType: 1 INT8, 3 FP32, 4 INT32. */
int64_t cim22_cuda_model_num_inputs(const cim22_cuda_model *model);
int64_t cim22_cuda_model_num_outputs(const cim22_cuda_model *model);
int64_t cim22_cuda_model_rank(const cim22_cuda_model *model, int64_t tensor);
int64_t cim22_cuda_model_dim(const cim22_cuda_model *model, int64_t tensor, int64_t axis);
int64_t cim22_cuda_model_dtype(const cim22_cuda_model *model, int64_t tensor);
int64_t cim22_cuda_model_num_transactions(const cim22_cuda_model *model);
uint64_t cim22_cuda_model_dispatch_count(const cim22_cuda_model *model);
const char *cim22_cuda_model_error(const cim22_cuda_model *model);
/* Replaces cim22_session_invoke (runtime/Runtime.cpp:292-340): buffers are
 * host pointers to contiguous row-major tensors, inputs then outputs, with
 * counts[i] elements each; they are passed as MLIR ranked descriptors. Calls
 * on one model are serialized. Returns 0, or 1 with the diagnostic in
 * cim22_cuda_model_error ("runtime buffer count mismatch", "runtime buffer
 * element count mismatch", or "kernel: <runner error>"). */
int cim22_cuda_model_invoke(cim22_cuda_model *model, void **buffers, const int64_t *counts,
                            int64_t num_buffers);

/* ------------------------------------------------------------------------ */
/* 3. Layer level, device memory, stream ordered.
 *
 * A CIM layer is a contraction y[m, n] = sum_k W[n, k] x[m, k] executed as the
 * compiler tiles it: 16-lane N tiles, 64-element K tiles with zero padding
 * (Passes.cpp:760-826), one crossbar Work per (column m, N tile, K tile).
 *
 * Status words: kernels OR error bits (CIM22_STATUS_*) into a caller-owned
 * device int32. The word is read after the stream is synchronized; the
 * message of each bit is returned by cim22_cuda_status_message. */

#define CIM22_STATUS_INPUT_NOT_FINITE 0x1   /* NaN/Inf reached a BF16 tile input */
#define CIM22_STATUS_TILE_OVERFLOW 0x2      /* compensated tile exceeds BF16 */
#define CIM22_STATUS_I21_RANGE 0x4          /* INT8 partial outside signed i21 */
#define CIM22_STATUS_NORMALIZATION 0x8      /* sign-split prealign invariant broken */
#define CIM22_STATUS_BAD_ARGUMENT 0x10      /* launch-time argument check failed */
#define CIM22_STATUS_NEGATIVE_INPUT 0x20    /* negative value in a nonnegative (2-branch) layer */
#define CIM22_STATUS_TIMEOUT 0x40           /* a bounded on-device wait gave up (results invalid) */
#define CIM22_STATUS_CHIP_NOT_FINITE 0x80   /* Legacy: a chip output to compensate is not finite */
#define CIM22_STATUS_LEGACY_SCALING 0x100   /* Legacy group scaling changed prealigned mantissas */
#define CIM22_STATUS_LEGACY_I21 0x200       /* Legacy: all -128 input group and weight lane */

/* Message of the lowest set status bit ("" for 0). */
const char *cim22_cuda_status_message(int32_t status);

/* Diagnostic of the last failing layer or glue call on this thread. */
const char *cim22_cuda_last_error(void);

/* Number of tcgen05 tensor-core kernel launches issued by this process so
 * far (diagnostics: shows which contraction path a layer took). */
int64_t cim22_cuda_tensor_core_launches(void);

/* No counterpart in the reference. Self-check of the bounded on-device wait
 * that every tensor-core pipeline uses for its mbarriers: one CTA waits on a
 * barrier that nothing completes, gives up after limit_ns nanoseconds of the
 * GPU's global timer and ORs CIM22_STATUS_TIMEOUT into *status (a device
 * int32). The kernel holds no TMEM and issues no copies, so the context stays
 * usable. Returns 0, or CIM22_STATUS_BAD_ARGUMENT for a null status or a
 * limit outside (0, 10 s]. Asynchronous on `stream`. */
int cim22_cuda_check_wait_timeout(uint64_t limit_ns, int32_t *status, void *stream);

/* sizeof of each structure above, in declaration order: frame_packet,
 * static_weight, input_binding, readback_binding, work, group, transaction,
 * trace_event, memref2d, gather. Returns the number of entries written. */
int cim22_cuda_abi_sizes(int64_t *sizes, int capacity);

typedef struct cim22_cuda_layer cim22_cuda_layer;

/* BF16 sign-split weights. weight is a host f32 [n, k] matrix (row = output
 * lane, k in the reduction order of the lowered op). Per Passes.cpp:2304-2476
 * the weights are split into Wp = max(W, 0) and Wn = max(-W, 0), rounded to
 * BF16 with round-to-nearest-even and prealigned per (16-lane, 64-K) tile and
 * lane (BF16Support.cpp:56-70), then kept resident in device memory.
 * Non-finite weights are rejected ("BF16 correction requires finite fixed
 * weights", Passes.cpp:2349-2352). */
cim22_cuda_layer *cim22_cuda_layer_create_bf16(int device, const float *weight,
                                               int64_t n, int64_t k,
                                               char *error,
                                               size_t error_capacity);

/* INT8 weights, host int8 [n, k]. The per-(lane, K tile) signed-i21 range
 * proof over every int8 input (Passes.cpp:592-627) is evaluated at creation;
 * cim22_cuda_layer_range_safe reports it. Proven layers accumulate the whole
 * K range exactly in int32; unproven layers run the checked per-tile kernel
 * that reports CIM22_STATUS_I21_RANGE. */
cim22_cuda_layer *cim22_cuda_layer_create_int8(int device, const int8_t *weight,
                                               int64_t n, int64_t k,
                                               char *error,
                                               size_t error_capacity);
void cim22_cuda_layer_destroy(cim22_cuda_layer *layer);
int cim22_cuda_layer_range_safe(const cim22_cuda_layer *layer);
/* 1 when a BF16 sign-split layer takes BF16 operands: at least 64 output
 * lanes, and every lane with a nonzero mantissa has a weight exponent in
 * [8, 241]. On sm_100 its prepare then stores scaled BF16 operand values
 * (twice the workspace bytes of int8 mantissas) and its contraction runs the
 * tensor-core kernel with BF16 operands; 0 otherwise (int8 mantissas and the
 * int8 tensor-core kernel). No counterpart in the reference: the operand
 * format is internal to this backend and the outputs are the same. */
int cim22_cuda_layer_bf16_operands(const cim22_cuda_layer *layer);
int64_t cim22_cuda_layer_n(const cim22_cuda_layer *layer);
int64_t cim22_cuda_layer_k(const cim22_cuda_layer *layer);

/* Epilogue activations fused into the layer kernel. */
#define CIM22_ACT_NONE 0
#define CIM22_ACT_RELU 1
#define CIM22_ACT_GELU 2

/* Gather descriptor of the K x columns operand. Linear: x is [m, k] row-major.
 * Conv (im2col, Passes.cpp:1087-1385): x is an image batch; column m =
 * (n, oh, ow), K index = c*kh*kw + i*kw + j (the FCHW weight order), zero
 * padding inside 64-element groups. A Linear applied to torch.flatten of an
 * NHWC image is the conv gather whose kernel covers the whole image
 * (out 1x1): K index c*H*W + h*W + w is exactly the NCHW flatten order. */
#define CIM22_GATHER_ROWS 0
#define CIM22_GATHER_CONV_NCHW 1
#define CIM22_GATHER_CONV_NHWC 2

typedef struct cim22_gather {
  int32_t kind;
  int32_t batch, channels, height, width; /* image geometry (conv only) */
  int32_t kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w;
  int32_t out_h, out_w;
  /* Optional max pooling folded into a conv gather (either layout): when
   * pool_kernel > 0, x is the pre-pool image of pool_src_h x pool_src_w and
   * the conv reads max over each pool_kernel^2 window (stride pool_stride,
   * no padding), with height/width the pooled size. */
  int32_t pool_kernel, pool_stride, pool_src_h, pool_src_w;
} cim22_gather;

/* A BF16 layer in a given compensation mode (CIM22_BF16_SIGN_SPLIT is
 * cim22_cuda_layer_create_bf16). CIM22_BF16_LEGACY and CIM22_BF16_NONE are
 * the reference's diagnostic modes (compiler.py:25, bf16_compensation): no
 * sign split, signed prealigned tiles, the mode's input preparation and
 * restore (BF16Compensation.cpp:84-164); the branches argument of the
 * forward calls is ignored for them. */
cim22_cuda_layer *cim22_cuda_layer_create_bf16_mode(int device, const float *weight,
                                                    int64_t n, int64_t k, int32_t compensation,
                                                    char *error, size_t error_capacity);
/* The layer's CIM22_BF16_* compensation mode (-1 for a null layer). */
int32_t cim22_cuda_layer_compensation(const cim22_cuda_layer *layer);

/* Scratch bytes needed by cim22_cuda_layer_forward_bf16 for m columns. */
size_t cim22_cuda_layer_workspace_bf16(const cim22_cuda_layer *layer,
                                       int64_t m, int32_t branches);

/* BF16 sign-split layer: activation split into xp/xn, RNE to BF16, per-64
 * group normalisation and prealignment (BF16Compensation.cpp:84-137), one
 * 64x16 crossbar dot per (column, lane tile, K tile) with the per-tile
 * truncating converter and binary64-exact scale recovery
 * (BF16Compensation.cpp:33-51,149-164), f32 K accumulation in tile order,
 * BF16 rounding when more than one K tile, branch merge
 * ((pp - pn) - np) + nn in f32 (Passes.cpp:2405-2416), then + bias and the
 * activation. branches is 4, or 2 when the input is known nonnegative
 * (the xn branches are exactly +0 then). y is f32 [m, n] row-major; for conv
 * gathers that is NHWC. */
int cim22_cuda_layer_forward_bf16(const cim22_cuda_layer *layer, const float *x,
                                  const cim22_gather *gather, int64_t m,
                                  const float *bias, int32_t activation,
                                  int32_t branches, float *y, void *workspace,
                                  size_t workspace_bytes, int32_t *status,
                                  void *stream);

/* No counterpart in the reference. The same BF16 sign-split layer as
 * cim22_cuda_layer_forward_bf16 for callers that cannot allocate device
 * memory: generated model code that, like the reference's compiled Host code,
 * owns only stack buffers and has no device allocator, and embedders whose
 * device memory is owned and budgeted by another component. The
 * prepared-column scratch lives in a library-owned 16 MiB
 * __device__ array (held by every GPU that loads the library until exit);
 * calls needing more (cim22_cuda_layer_workspace_bf16 > that size) are
 * rejected with CIM22_STATUS_BAD_ARGUMENT and a message in
 * cim22_cuda_last_error(). All calls on a device share the array: calls that
 * overlap on the GPU race. The layer's device must be current; the first call
 * on a device resolves the array's address and should precede any stream
 * capture. Allocates nothing. */
int cim22_cuda_layer_forward_bf16_noalloc(const cim22_cuda_layer *layer,
                                          const float *x,
                                          const cim22_gather *gather, int64_t m,
                                          const float *bias,
                                          int32_t activation, int32_t branches,
                                          float *y, int32_t *status,
                                          void *stream);
/* Size of that static scratch in bytes. */
size_t cim22_cuda_layer_noalloc_scratch_bytes(void);

/* Scratch bytes needed by cim22_cuda_layer_forward_int8 for m columns. */
size_t cim22_cuda_layer_workspace_int8(const cim22_cuda_layer *layer,
                                       int64_t m);

/* The two kernels of cim22_cuda_layer_forward_bf16, callable separately:
 * prepare gathers, splits and prealigns the activation columns into the
 * workspace; contract runs the crossbar dots, restore, K accumulation, branch
 * merge, bias and activation from that workspace. forward = prepare then
 * contract on the same stream. */
int cim22_cuda_layer_prepare_bf16(const cim22_cuda_layer *layer,
                                  const float *x, const cim22_gather *gather,
                                  int64_t m, int32_t branches, void *workspace,
                                  size_t workspace_bytes, int32_t *status,
                                  void *stream);
int cim22_cuda_layer_contract_bf16(const cim22_cuda_layer *layer, int64_t m,
                                   const float *bias, int32_t activation,
                                   int32_t branches, float *y,
                                   const void *workspace,
                                   size_t workspace_bytes, int32_t *status,
                                   void *stream);

/* No counterpart in the reference's C interface: the same layer with two
 * options for the code around it. y is written as NCHW images,
 * y[m / out_pixels][n][out_pixels], column m being (image, pixel) =
 * (m / out_pixels, m % out_pixels) - the layout of the conv output the
 * reference hands to the next torch op - when out_pixels > 0 (it must divide
 * m), or as [m, n] rows when out_pixels = 0. When post_scale and post_shift
 * are given (both or neither), each output becomes
 * fma(out, post_scale[n], post_shift[n]) after the bias and before the
 * activation: an inference batch norm that follows the layer, computed
 * exactly as cim22_cuda_channel_affine_* computes it. */
int cim22_cuda_layer_forward_bf16_ex(const cim22_cuda_layer *layer, const float *x,
                                     const cim22_gather *gather, int64_t m, int64_t out_pixels,
                                     const float *bias, const float *post_scale,
                                     const float *post_shift, int32_t activation,
                                     int32_t branches, float *y, void *workspace,
                                     size_t workspace_bytes, int32_t *status, void *stream);
/* 1 when cim22_cuda_layer_forward_bf16{,_ex} may run the layer as one kernel
 * that gathers, prealigns and contracts, so that its prepared columns never
 * leave the SM: one-tile layers (K <= 64) of at most 64 lanes (one thread per
 * column) and layers of at most 16 lanes and two K tiles (the CUDA-core
 * contraction building its own activation tiles). Such a call picks, by the
 * gather, output layout, branch count and column count, whichever was
 * measured faster on B200, running the prepare and contract kernels itself
 * where those win. 0: the caller runs prepare and contract. */
int cim22_cuda_layer_fused_forward(const cim22_cuda_layer *layer);
int cim22_cuda_layer_contract_bf16_ex(const cim22_cuda_layer *layer, int64_t m,
                                      int64_t out_pixels, const float *bias,
                                      const float *post_scale, const float *post_shift,
                                      int32_t activation, int32_t branches, float *y,
                                      const void *workspace, size_t workspace_bytes,
                                      int32_t *status, void *stream);
/* contract_bf16_ex with a residual add fused after the per-lane fma and
 * before the activation: y = act(fma(merge + bias, post_scale, post_shift) +
 * residual), one f32 add per element as the Host glue of a residual block
 * (Conv -> BatchNorm -> add -> ReLU) computes it. residual is laid out like y
 * (rows or NCHW planes, out_pixels as for y) and may be NULL. Sign-split
 * layers only. */
int cim22_cuda_layer_contract_bf16_res(const cim22_cuda_layer *layer, int64_t m,
                                       int64_t out_pixels, const float *bias,
                                       const float *post_scale, const float *post_shift,
                                       const float *residual, int32_t activation,
                                       int32_t branches, float *y, const void *workspace,
                                       size_t workspace_bytes, int32_t *status, void *stream);

/* INT8 layer: y[m, n] = sum over K tiles of the signed-i21 tile results,
 * accumulated in wrapping int32 (Passes.cpp:1054-1059). x is int8 [m, k]. */
int cim22_cuda_layer_forward_int8(const cim22_cuda_layer *layer,
                                  const int8_t *x, int64_t m, int32_t *y,
                                  void *workspace, size_t workspace_bytes,
                                  int32_t *status, void *stream);

/* INT8 layer with the compiler's INT8 Conv and bias lowerings
 * (Passes.cpp:1402-1557, 1863-2012, 2049-2155):
 *   gather      NULL or CIM22_GATHER_ROWS: x is int8 [m, k]. A conv gather
 *               (NCHW or NHWC, no fused pool): x is an int8 image batch and
 *               m = batch * out_h * out_w columns in (image, oh, ow) order,
 *               K in (channel, kh, kw) order (weights [F][C][KH][KW]).
 *   pad_bottom, pad_right
 *               bottom/right zero padding of a conv gather when it differs
 *               from pad_h/pad_w (ONNX ConvInteger pads); -1 = symmetric.
 *   bias        optional int32 [n], added with int32 wraparound. The
 *               compiler folds an int8-range bias into the crossbar as one
 *               more K column (weight = bias, input = 1) when the range proof
 *               allows, and leaves it as a Host add otherwise; both give this
 *               exact sum.
 *   out_pixels  0: y is [m, n]; > 0: y is NCHW [m / out_pixels][n][out_pixels].
 *   exact_unproven
 *               for weights that fail the i21 range proof: nonzero computes
 *               the exact wrapping int32 sum, as the compiler keeps such an
 *               op on the Host (Passes.cpp:592-627); zero runs the checked
 *               per-tile kernel that reports CIM22_STATUS_I21_RANGE.
 * Workspace: cim22_cuda_layer_workspace_int8(layer, m) bytes. */
int cim22_cuda_layer_forward_int8_ex(const cim22_cuda_layer *layer, const int8_t *x,
                                     const cim22_gather *gather, int64_t m, int32_t pad_bottom,
                                     int32_t pad_right, const int32_t *bias, int64_t out_pixels,
                                     int32_t exact_unproven, int32_t *y, void *workspace,
                                     size_t workspace_bytes, int32_t *status, void *stream);

/* A chain of small BF16 sign-split layers in one persistent kernel (no
 * counterpart in the reference's interface; the numerics are those of
 * cim22_cuda_layer_forward_bf16 layer by layer). Each CTA carries whole
 * images through every layer with the activations in shared memory: per
 * layer the im2col gather, split, prealign, crossbar dots, restore, tile
 * sums, merge, bias and activation, then an optional 2x2 stride-2 max pool.
 * Meant for networks whose per-image activations fit in shared memory
 * (LeNet-5, the MNIST MLP), where per-layer launches are latency-bound. */
#define CIM22_CHAIN_LINEAR 0
#define CIM22_CHAIN_CONV 1
typedef struct cim22_chain_layer {
  int32_t kind;                     /* CIM22_CHAIN_CONV or CIM22_CHAIN_LINEAR */
  const cim22_cuda_layer *layer;    /* sign-split weights [n][c * kh * kw] */
  const float *bias;                /* device [n] or NULL */
  /* First layer only: the input image [channels][height][width] (a vector
   * input is [k][1][1]); later layers take the previous output. A Linear
   * layer flattens its input in NCHW order. */
  int32_t channels, height, width;
  int32_t kernel_h, kernel_w, stride, pad; /* conv only */
  int32_t branches;                 /* 4, or 2 when the input is nonnegative */
  int32_t activation;               /* CIM22_ACT_* */
  int32_t pool;                     /* 0, or 2: 2x2 stride-2 max pool after it */
} cim22_chain_layer;
/* x: f32 [batch][input image]; y: f32 [batch][last output, NCHW order]. */
int cim22_cuda_chain_forward(const cim22_chain_layer *layers, int32_t n_layers, const float *x,
                             int64_t batch, float *y, int32_t *status, void *stream);

/* ------------------------------------------------------------------------ */
/* Host glue the compiler emits around CIM layers (upstream Linalg lowering,
 * lib/Compiler/Pipelines.cpp:61-72). All f32, device memory; image layout
 * in the function name. */

int cim22_cuda_relu(const float *x, float *y, int64_t count, void *stream);
int cim22_cuda_add(const float *a, const float *b, float *y, int64_t count,
                   int32_t activation, void *stream);
int cim22_cuda_gelu(const float *x, float *y, int64_t count, void *stream);
/* Max/average pooling over an NHWC batch (no padding when pad = 0; average
 * pooling divides by the full window, count_include_pad semantics). */
int cim22_cuda_maxpool2d_nhwc(const float *x, float *y, int32_t n, int32_t h,
                              int32_t w, int32_t c, int32_t kernel,
                              int32_t stride, int32_t pad, void *stream);
int cim22_cuda_avgpool2d_nhwc(const float *x, float *y, int32_t n, int32_t h,
                              int32_t w, int32_t c, int32_t kernel,
                              int32_t stride, void *stream);
/* Mean over H and W of an NHWC batch -> [n, c]. */
int cim22_cuda_global_avgpool_nhwc(const float *x, float *y, int32_t n,
                                   int32_t h, int32_t w, int32_t c,
                                   void *stream);
/* Per-channel affine y = x * scale[c] + shift[c] (+ activation), NHWC. */
int cim22_cuda_channel_affine_nhwc(const float *x, const float *scale,
                                   const float *shift, float *y, int64_t rows,
                                   int32_t c, int32_t activation, void *stream);
/* Row softmax over the last dimension of [rows, cols]. */
int cim22_cuda_softmax(const float *x, float *y, int64_t rows, int32_t cols,
                       void *stream);
/* NHWC [n, h, w, c] -> NCHW-flattened [n, c*h*w] (torch.flatten order). */
int cim22_cuda_nhwc_to_nchw(const float *x, float *y, int32_t n, int32_t h,
                            int32_t w, int32_t c, void *stream);
/* NCHW -> NHWC. */
int cim22_cuda_nchw_to_nhwc(const float *x, float *y, int32_t n, int32_t c,
                            int32_t h, int32_t w, void *stream);
/* Elementwise f32 glue (Host arithmetic around the layers, e.g. the LIF
 * membrane updates of spiking models, python/tests/test_backend.py:502-545):
 * y[i] = a[i] op b[i], where a NULL a or b stands for the scalar a_scalar /
 * b_scalar. One IEEE round-to-nearest operation per element, as PyTorch's
 * CPU kernels compute it; comparisons give 1.0f or 0.0f (0 for NaN); max/min
 * propagate NaN like torch.maximum/minimum. y may alias a or b. */
#define CIM22_BINARY_ADD 0
#define CIM22_BINARY_SUB 1
#define CIM22_BINARY_MUL 2
#define CIM22_BINARY_DIV 3
#define CIM22_BINARY_GE 4
#define CIM22_BINARY_GT 5
#define CIM22_BINARY_LE 6
#define CIM22_BINARY_LT 7
#define CIM22_BINARY_EQ 8
#define CIM22_BINARY_NE 9
#define CIM22_BINARY_MAX 10
#define CIM22_BINARY_MIN 11
int cim22_cuda_binary(const float *a, const float *b, float *y, int64_t count, int32_t op,
                      float a_scalar, float b_scalar, void *stream);
/* y[i] = value. */
int cim22_cuda_fill(float *y, int64_t count, float value, void *stream);
/* Copies `words` 32-bit words (slice writes and state updates). */
int cim22_cuda_copy(const void *src, void *dst, int64_t words, void *stream);
/* Copies `blocks` runs of `inner` 32-bit words; run b is read at
 * src + b * src_stride and written at dst + b * dst_stride (words). Selecting
 * index i of axis d of a contiguous tensor is blocks = prod(shape[:d]),
 * inner = prod(shape[d+1:]), src offset i * inner, src_stride =
 * shape[d] * inner; select_scatter writes the same runs the other way. */
int cim22_cuda_slice_copy(const void *src, void *dst, int64_t blocks, int64_t inner,
                          int64_t src_stride, int64_t dst_stride, void *stream);
/* No counterpart in the reference (it runs on one host): reassembles a
 * layer whose output lanes are split over `ranks` devices. src is what an
 * all-gather of the per-rank [rows][cols] outputs stacks, [ranks][rows][cols];
 * dst is [rows][total] with rank r's block in columns r*cols .. r*cols+cols-1
 * (trailing blocks may be padded: columns at or past total are dropped). */
int cim22_cuda_unshard_columns(const float *src, float *dst, int32_t ranks, int64_t rows,
                               int64_t cols, int64_t total, void *stream);
/* No counterpart in the reference (it runs on one host): peer memory for a
 * layer whose output lanes are split over the GPUs of one node, so that the
 * contraction's epilogue writes each rank's lane block straight into every
 * rank's full output over NVLink (the compute step and the all-gather in one
 * kernel), and a device-side barrier orders the layers.
 *
 * cim22_cuda_device_alloc returns zero-filled device memory of its own
 * cudaMalloc (an IPC handle covers a whole allocation, so buffers to share
 * are allocated here); cim22_cuda_ipc_get_handle writes the
 * CIM22_IPC_HANDLE_BYTES-byte handle of such a buffer, and another process
 * on the same node maps it with cim22_cuda_ipc_open_handle (peer access
 * enabled lazily) and unmaps it with cim22_cuda_ipc_close_handle. */
#define CIM22_IPC_HANDLE_BYTES 64
#define CIM22_MAX_PEERS 8
int cim22_cuda_device_alloc(size_t bytes, void **ptr);
int cim22_cuda_device_free(void *ptr);
int cim22_cuda_ipc_get_handle(const void *base, void *handle);
int cim22_cuda_ipc_open_handle(const void *handle, void **base);
int cim22_cuda_ipc_close_handle(void *base);

/* Where a column-sharded layer's outputs go: out[p] is rank p's full
 * [rows][row_stride] f32 output as mapped on this device (out[rank] the
 * local one); this rank's lanes land in columns lane_offset .. lane_offset +
 * lanes - 1 of every out[p] (the layer's further lanes are padding and are
 * not stored). */
typedef struct cim22_peer_outputs {
  float *out[CIM22_MAX_PEERS];
  int32_t ranks;
  int64_t row_stride;
  int64_t lane_offset;
  int64_t lanes;
} cim22_peer_outputs;

/* cim22_cuda_layer_contract_bf16 for a layer with BF16 operands
 * (cim22_cuda_layer_bf16_operands) whose outputs are rows: the epilogue
 * stores every output value into all peers' buffers of `peers` (float4
 * stores where row_stride, lane_offset and the buffers allow) and makes
 * them visible system-wide before the kernel ends. Prepare with
 * cim22_cuda_layer_prepare_bf16 into the same workspace first. */
int cim22_cuda_layer_contract_bf16_peers(const cim22_cuda_layer *layer, int64_t m,
                                         const float *bias, int32_t activation,
                                         int32_t branches, const cim22_peer_outputs *peers,
                                         const void *workspace, size_t workspace_bytes,
                                         int32_t *status, void *stream);

/* A barrier of `ranks` GPUs in one launch per rank: flags[p] is rank p's
 * array of ranks + 1 int32 words (zero-filled at allocation) as mapped on
 * this device. One thread raises this rank's epoch (the last word of its own
 * array), makes every earlier write of the stream visible system-wide,
 * stores the epoch into word `rank` of every rank's array and waits until
 * every word of its own array holds at least that epoch. A wait that runs
 * out after limit_ns of the GPU's global timer ORs CIM22_STATUS_TIMEOUT into
 * *status and returns (the outputs of the step are then invalid). Every rank
 * makes the same sequence of barrier calls. */
typedef struct cim22_peer_flags {
  int32_t *flags[CIM22_MAX_PEERS];
  int32_t ranks;
  int32_t rank;
} cim22_peer_flags;
int cim22_cuda_peer_barrier(const cim22_peer_flags *flags, uint64_t limit_ns, int32_t *status,
                            void *stream);

/* The pooling and affine glue on NCHW batches [n, c, h, w]. */
int cim22_cuda_maxpool2d_nchw(const float *x, float *y, int32_t n, int32_t c,
                              int32_t h, int32_t w, int32_t kernel,
                              int32_t stride, int32_t pad, void *stream);
int cim22_cuda_avgpool2d_nchw(const float *x, float *y, int32_t n, int32_t c,
                              int32_t h, int32_t w, int32_t kernel,
                              int32_t stride, void *stream);
/* Mean over H and W -> [n, c]. */
int cim22_cuda_global_avgpool_nchw(const float *x, float *y, int32_t n,
                                   int32_t c, int32_t h, int32_t w,
                                   void *stream);
/* y = x * scale[c] + shift[c] (+ activation) for planes of hw elements. */
int cim22_cuda_channel_affine_nchw(const float *x, const float *scale,
                                   const float *shift, float *y, int32_t n,
                                   int32_t c, int64_t hw, int32_t activation,
                                   void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CIM22_CUDA_H */
