/*
 * eir_cuda.h -- C-ABI of the einsum_ir B200 backend (sm_100a).
 *
 * This is the only boundary between host code and the CUDA kernels. Every entry
 * point is `extern "C"`, takes plain pointers and sizes, returns an int status
 * (values mirror einsum_ir::err_t, src/constants.h:33-46 of the reference) and
 * never throws. Device pointers are owned by the caller. Calls that take a
 * stream are asynchronous on that stream (a `void*` holding a cudaStream_t;
 * NULL = the legacy default stream). Plans are immutable after creation and
 * may be used from several host threads on different streams, except where a
 * plan owns a workspace (eir_plan_workspace_bytes() > 0): such a plan must not
 * run on two streams at once.
 *
 * Reference interfaces replaced (paths inside scalable-analyses/einsum_ir):
 *   eir_contract_plan_create  <- backend::BinaryContraction::init + compile
 *                                (src/backend/BinaryContraction.h:326-362)
 *   eir_contract              <- backend::BinaryContraction::contract
 *                                (src/backend/BinaryContraction.h:371-386)
 *   eir_permute_plan_create   <- backend::Unary::init + compile (src/backend/Unary.h:98-146)
 *   eir_permute               <- backend::Unary::eval (src/backend/Unary.h:148-156)
 *   eir_expression_*          <- frontend::EinsumExpression init/compile/eval/num_ops
 *                                (src/frontend/EinsumExpression.h:148-208)
 *   eir_contract_num_ops      <- backend::BinaryContraction::num_ops (BinaryContraction.h:391)
 */
#ifndef EIR_CUDA_H
#define EIR_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes: identical values to einsum_ir::err_t */
enum {
  EIR_SUCCESS                   = 0,
  EIR_COMPILATION_FAILED        = 1,
  EIR_DIMENSION_ORDERING_FAILED = 2,
  EIR_TENSOR_BLOCKING_FAILED    = 3,
  EIR_NO_DATA_PTR_PROVIDED      = 4,
  EIR_CALLED_BEFORE_COMPILATION = 5,
  EIR_INVALID_ID                = 6,
  EIR_INVALID_BACKEND           = 7,
  EIR_INVALID_CPX_DIM           = 8,
  EIR_INVALID_DTYPE             = 9,
  EIR_INVALID_KTYPE             = 10,
  EIR_CUDA_ERROR                = 50, /* extension: a CUDA runtime/driver call failed */
  EIR_DEVICE_TIMEOUT            = 51, /* extension: a bounded device-side wait gave up */
  EIR_INVALID_ARGUMENT          = 52, /* extension: null plan / bad descriptor */
  EIR_UNDEFINED_ERROR           = 99
};

/* dimension types: identical values to einsum_ir::dim_t (C, M, N, K, CPX).
 * EIR_DIM_CPX: the complex dimension (size 2: real, imaginary part) of a
 * complex contraction, present in left, right and out (dim_t::CPX,
 * src/constants.h:13); it needs ktype_main EIR_KTYPE_CPX_MADD. */
enum { EIR_DIM_C = 0, EIR_DIM_M = 1, EIR_DIM_N = 2, EIR_DIM_K = 3, EIR_DIM_CPX = 4 };

/* data types: FP32/FP64 keep einsum_ir::data_t values; BF16 is an extension */
enum { EIR_FP32 = 0, EIR_FP64 = 1, EIR_BF16 = 2, EIR_UNDEFINED_DTYPE = 99 };

/* compute types (extension; the reference computes in the data type) */
enum {
  EIR_COMPUTE_DEFAULT = 0, /* FP32 data -> FP32-exact (3xTF32 or SIMT FP32); FP64 -> FP64; BF16 -> FP32 acc */
  EIR_COMPUTE_FP32    = 1, /* FP32-accurate result (error ~1e-6 relative) */
  EIR_COMPUTE_TF32    = 2, /* single TF32 tensor-core pass, FP32 accumulate */
  EIR_COMPUTE_FP64    = 3,
  EIR_COMPUTE_BF16    = 4  /* BF16 multiplicands, FP32 accumulate */
};

/* kernel types: identical values to einsum_ir::kernel_t (the real kernels and
 * the complex zero / multiply-add pair, src/constants.h:60-76) */
enum {
  EIR_KTYPE_ZERO = 0, EIR_KTYPE_RELU = 1, EIR_KTYPE_ADD = 2, EIR_KTYPE_COPY = 3,
  EIR_KTYPE_MADD = 4, EIR_KTYPE_CPX_ZERO = 6, EIR_KTYPE_CPX_MADD = 8, EIR_KTYPE_UNDEFINED = 99
};

/* kernel family chosen by the planner (eir_plan_kernel_family) */
enum {
  EIR_FAMILY_NONE      = 0,
  EIR_FAMILY_SIMT      = 1, /* generic strided CUDA-core contraction */
  EIR_FAMILY_TC        = 2, /* tcgen05 + TMA tensor-core contraction */
  EIR_FAMILY_PERMUTE   = 3, /* permute kernel */
  EIR_FAMILY_DMMA      = 4  /* FP64 tensor-core (mma.sync f64) contraction */
};

/* planner flags */
enum {
  EIR_FLAG_FORCE_SIMT   = 1, /* never use the tensor-core path */
  EIR_FLAG_NO_PREPACK   = 2  /* never pre-permute an operand into the workspace */
};

/* one loop dimension of a binary contraction; strides are in ELEMENTS.
 * A stride of 0 means the tensor does not depend on the dimension (e.g. an
 * aux bias broadcast, the reference's "outer size 1" convention). */
typedef struct {
  int32_t type;            /* EIR_DIM_* */
  int32_t pad_;
  int64_t size;
  int64_t stride_left;
  int64_t stride_right;
  int64_t stride_out;
  int64_t stride_out_aux;
} eir_dim;

typedef struct {
  int32_t        num_dims;
  int32_t        dtype_left;   /* EIR_FP32 / EIR_FP64 / EIR_BF16 */
  int32_t        dtype_right;
  int32_t        dtype_out;    /* EIR_FP32 / EIR_FP64 */
  int32_t        dtype_comp;   /* EIR_COMPUTE_* */
  int32_t        ktype_first_touch; /* ZERO, COPY, ADD or UNDEFINED */
  int32_t        ktype_main;        /* MADD */
  int32_t        ktype_last_touch;  /* RELU, ADD or UNDEFINED */
  int32_t        flags;             /* EIR_FLAG_* */
  int32_t        pad_;
  eir_dim const *dims;
} eir_contract_desc;

typedef struct eir_plan eir_plan;
typedef struct eir_expression eir_expression;

/* --- binary contraction ------------------------------------------------ */
int     eir_contract_plan_create(eir_contract_desc const *desc, eir_plan **plan);
/* out_aux may be NULL when no touch kernel reads it */
int     eir_contract(eir_plan *plan, void const *left, void const *right,
                     void const *out_aux, void *out, void *stream);
int64_t eir_contract_num_ops(eir_plan const *plan);
/* Same contraction as eir_contract, but allocates no device memory: for
 * callers whose device memory is owned by another allocator (a framework's
 * caching allocator, a serving arena) or that cannot afford cudaMalloc's
 * synchronisation on the hot path. A plan's pre-permute scratch comes from a
 * static 8 MiB array in the library's device image (held on every GPU that
 * loads the library); plans needing more are rejected with
 * EIR_INVALID_ARGUMENT. The first call on a device does a one-time set-up
 * (make it before any stream capture). All calls share the array: calls that
 * overlap on the GPU race. No counterpart in the reference. */
int     eir_contract_no_alloc(eir_plan *plan, void const *left, void const *right,
                              void const *out_aux, void *out, void *stream);

/* Same contraction as eir_contract, and every final output element is also
 * stored, at the same element offset, into each of num_peers (<= 7) other
 * output buffers: typically the outputs of the other GPUs of a batch-sharded
 * contraction, mapped into this process with eir_ipc_open_handle, so that
 * the all-gather of the output happens inside the contraction's epilogue
 * (plain stores over NVLink, overlapped with the next tiles) instead of a
 * separate collective. The peer buffers must have out's layout and extent.
 * Their contents are complete when the call's kernels have completed; a
 * reader on another GPU synchronises with this stream first (e.g. a
 * cross-process barrier after a stream synchronisation). Not for complex
 * plans. No counterpart in the reference (it has no multi-GPU path). */
int     eir_contract_peers(eir_plan *plan, void const *left, void const *right,
                           void const *out_aux, void *out, int32_t num_peers,
                           void *const *peer_outs, void *stream);

/* Same contraction as eir_contract, followed by the all-gather step of a
 * sharded contraction: the finished output is copied, at the same byte
 * offsets, into each of num_peers (<= 7) other buffers of out's extent
 * (typically this rank's block inside the full outputs of the other GPUs,
 * mapped with eir_ipc_open_handle). The copies run on the copy engines, one
 * stream per peer owned by the plan, so they take no SM from the
 * contraction. When the output's outermost dim is the kernel's slowest tile
 * loop and the kernel publishes per-slab completion (FP64 plans on the DMMA
 * kernel), the copy of each slab of that dim starts as soon as the kernel has
 * stored it, overlapping the slabs still being computed; otherwise the
 * copies start when the kernel ends. The output must be one contiguous
 * block. Asynchronous on `stream`: once `stream` has passed the call, the
 * output and every peer copy are complete; a reader on another GPU first
 * synchronises with this rank (e.g. a stream synchronisation, then a
 * cross-process barrier). Like every workspace-owning plan, one plan must
 * not run on two streams at once. Not for complex plans. The copy streams
 * wait on the kernel's slab counters: run the process with
 * CUDA_DEVICE_MAX_CONNECTIONS >= 16 (set before its CUDA context exists), or
 * with CUDA's default of 8 hardware queues the waiting streams share queues
 * with the compute stream and with one another and hold back the work
 * behind them. No counterpart in the reference (it has no multi-GPU path;
 * BASELINE config 5 shards its batch dim z across GPUs and all-gathers the
 * output). */
int     eir_contract_gather(eir_plan *plan, void const *left, void const *right,
                            void const *out_aux, void *out, int32_t num_peers,
                            void *const *peer_outs, void *stream);

/* CUDA IPC of device buffers between the processes of one node (one process
 * per GPU): a handle (EIR_IPC_HANDLE_BYTES opaque bytes) and offset for a
 * pointer into any cudaMalloc'd allocation; the opening process gets the
 * pointer (mapped with peer access) and the mapping's base for closing. */
enum { EIR_IPC_HANDLE_BYTES = 64 };
/* copies `bytes` from src to each of num_peers destinations (typically peer
 * buffers mapped with eir_ipc_open_handle), one asynchronous copy-engine copy
 * per destination on `stream`: the gather step of a sharded contraction
 * that overlaps the next block's kernels without taking SMs from them */
int     eir_copy_to_peers(void const *src, int32_t num_peers, void *const *dsts, int64_t bytes,
                          void *stream);
int     eir_ipc_get_handle(void const *dev_ptr, void *handle, int64_t *offset);
int     eir_ipc_open_handle(void const *handle, int64_t offset, void **dev_ptr, void **base);
int     eir_ipc_close_handle(void *base);

/* --- output group of a sharded contraction (one process per GPU) ---------- */
/* The caller's exchange between the ranks: every rank passes `bytes` bytes in
 * `send` and receives all ranks' contributions, in rank order, in `recv`
 * (world * bytes). Any transport works (MPI_Allgather, NCCL on a device
 * buffer, sockets, torch.distributed); return 0 on success. */
typedef int (*eir_allgather_fn)(void const *send, void *recv, int64_t bytes, void *user);
typedef struct eir_output_group eir_output_group;
/* Maps the full output buffer `out` of every rank of a node into this
 * process (CUDA IPC handles exchanged with `allgather`; collective: every
 * rank calls it with its own buffer of the same size). Fails on every rank
 * (EIR_CUDA_ERROR) if some rank cannot export or map the buffers. No
 * counterpart in the reference (it has no multi-GPU path). */
int     eir_output_group_create(int32_t rank, int32_t world, void *out, eir_allgather_fn allgather,
                                void *user, eir_output_group **group);
/* the addresses, in the other ranks' buffers (rank order, this rank left
 * out: world - 1 entries), that correspond to byte `offset` of this rank's
 * buffer: the peer list of eir_contract_gather for the block at `offset` */
int     eir_output_group_peers(eir_output_group const *group, int64_t offset, void **peers);
/* closes the mappings; every rank destroys its group before any rank frees
 * its output buffer (e.g. a barrier between the two) */
int     eir_output_group_destroy(eir_output_group *group);

/* --- unary permute (copy with reordered strides) ------------------------- */
/* sizes/strides are per dimension, in elements; any order */
int     eir_permute_plan_create(int32_t num_dims, int64_t const *sizes,
                                int64_t const *strides_in, int64_t const *strides_out,
                                int32_t dtype, eir_plan **plan);
int     eir_permute(eir_plan *plan, void const *in, void *out, void *stream);
/* unary plan with the reference's kernel type: EIR_KTYPE_COPY (= the permute
 * above) or EIR_KTYPE_ZERO (out = 0 over strides_out; strides_in unused and
 * eir_permute's `in` may be NULL). Replaces basic::UnaryBackend::init +
 * compile with ktype_main COPY / ZERO (src/basic/unary/UnaryBackend.h:83-116,
 * eval :125). */
int     eir_unary_plan_create(int32_t num_dims, int64_t const *sizes,
                              int64_t const *strides_in, int64_t const *strides_out,
                              int32_t dtype, int32_t ktype, eir_plan **plan);

/* --- plans -------------------------------------------------------------- */
int     eir_plan_destroy(eir_plan *plan);
int     eir_plan_kernel_family(eir_plan const *plan);
/* bytes of device workspace the plan owns (pre-permuted operand), 0 if none */
int64_t eir_plan_workspace_bytes(eir_plan const *plan);
/* short human-readable description of the lowering (static storage per plan) */
char const *eir_plan_describe(eir_plan const *plan);

/* --- einsum expression (tree of binary contractions) -------------------- */
/* expr: "iae,bf,dcba,cg,dh->hgfei" (single-char) or "[a,b],[b,c]->[a,c]"
 * sizes: "32,8,4,2,16,64,8,8,8" in sorted-dim-name order (numeric-aware)
 * path:  "(1,2),(2,3),(0,1),(0,1)" (opt_einsum pair format)
 * dtype: EIR_FP32 / EIR_FP64 / EIR_BF16 (BF16: inputs BF16, intermediates/out FP32) */
int     eir_expression_create(char const *expr, char const *sizes, char const *path,
                              int32_t dtype, int32_t dtype_comp, eir_expression **expr_out);
/* ptrs: one device pointer per input tensor followed by the output pointer */
int     eir_expression_eval(eir_expression *expr, void *const *ptrs, void *stream);
int64_t eir_expression_num_ops(eir_expression const *expr);
int     eir_expression_num_tensors(eir_expression const *expr);  /* inputs + output */
int     eir_expression_tensor_dims(eir_expression const *expr, int32_t tensor,
                                   int64_t *sizes_out, int32_t max_dims);
int     eir_expression_destroy(eir_expression *expr);
char const *eir_expression_describe(eir_expression const *expr);

/* --- kernel timing (diagnostics) ------------------------------------------ */
/* enable: record CUDA events around the plan's main kernel on every call
 * (the pre-permute of a workspace operand is not included) */
int     eir_plan_profile(eir_plan *plan, int32_t enable);
/* synchronizes on the recorded events, returns the summed main-kernel time in
 * milliseconds and the number of timed launches, then clears the record */
int     eir_plan_profile_read(eir_plan *plan, double *ms_total, int64_t *launches);

/* --- errors / diagnostics ----------------------------------------------- */
char const *eir_last_error_string(void);
/* reads and clears the device-side error word of the current device
 * (set by bounded waits that gave up); synchronizes the stream */
int     eir_check_device_errors(void *stream);
/* number of kernels this library launched since load (all devices) */
int64_t eir_launch_count(void);
int     eir_version(void);

#ifdef __cplusplus
}
#endif

#endif /* EIR_CUDA_H */
