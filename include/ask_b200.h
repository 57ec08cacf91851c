/*
 * ask_b200.h -- C ABI of the B200 (sm_100a) kernel library for ASK's
 * data-parallel hot path: fused multi-output elementwise loops, reductions
 * (sum/prod/max/min/any/all/argmax/argmin), gather and scatter_add.
 *
 * The library replaces the owned-step kernels that ASK's CUDA lowering emits
 * (lib/Lowering/CUDA.cpp:152-419) and the launch those kernels get from the
 * Runtime's step launcher (lib/Runtime/CUDA.cpp:360-371).  A "plan" is one
 * owned execution-plan step: its ports are ordered inputs first, then outputs,
 * exactly as the reference kernel's pointer ABI and artifact port_map
 * (lib/Lowering/CUDA.cpp:177-208, schemas/execution-plan-v1.schema.json).
 *
 * Conventions
 *   - Every entry point returns an int status: 0 on success, a negative
 *     ASK_B200_E_* code otherwise; ask_b200_last_error() then returns a
 *     thread-local message.  No C++ exception crosses this boundary.  The
 *     reference Runtime wraps a failed driver call into CUDAError
 *     (lib/Runtime/CUDA.cpp:156-162); callers map non-zero statuses the same way.
 *   - Ports and scratch are caller-owned device memory.  A plan owns only
 *     immutable host metadata, so one plan may be launched concurrently on
 *     different streams with distinct scratch buffers.
 *   - Launches are stream-ordered: they enqueue kernels on the given stream,
 *     never synchronise, never allocate and never call back into the host,
 *     so they can be recorded into CUDA graphs by the caller.  The caller's
 *     current device must be the plan's device; launches change no device or
 *     context state (the reference pushes the context itself,
 *     lib/Runtime/CUDA.cpp:172-178).
 */
#ifndef ASK_B200_H
#define ASK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ASK_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define ASK_B200_API __attribute__((visibility("default")))
#else
#define ASK_B200_API
#endif

#define ASK_B200_OK 0
#define ASK_B200_E_INVALID (-1)     /* malformed recipe, bad argument, alignment */
#define ASK_B200_E_UNSUPPORTED (-2) /* a valid ASK step this library has no kernel for */
#define ASK_B200_E_CUDA (-3)        /* CUDA runtime error (message has the CUDA string) */
#define ASK_B200_E_NCCL (-4)        /* NCCL unavailable or a collective failed */
#define ASK_B200_E_DEVICE (-5)      /* no usable sm_100 device, or wrong current device */
#define ASK_B200_E_TIMEOUT (-6)     /* a bounded wait for other ranks ran out (ask_b200_comm_status) */

typedef struct ask_b200_plan ask_b200_plan;
typedef struct ask_b200_comm ask_b200_comm;

/* ABI version (ASK_B200_ABI_VERSION). */
ASK_B200_API int ask_b200_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
ASK_B200_API const char *ask_b200_last_error(void);

/*
 * Validate a recipe and build a plan for `device`.  Replaces ask::lowerToCUDALLVM
 * (lib/Lowering/CUDA.cpp:152) plus Session::load (lib/Runtime/CUDA.cpp:499-546)
 * for owned steps: the recipe names the step's family (elementwise, reduce,
 * gather, scatter_add), port types and static sizes, and its op program.
 * device = -1 builds a host-only plan (validation and describe only; launching
 * it fails), which needs no GPU.
 */
ASK_B200_API int ask_b200_plan_create(const char *recipe_json, int device, ask_b200_plan **out);
ASK_B200_API int ask_b200_plan_destroy(ask_b200_plan *plan);

/* Number of input and output ports (the reference's port_map order). */
ASK_B200_API int ask_b200_plan_ports(const ask_b200_plan *plan, size_t *n_inputs, size_t *n_outputs);

/*
 * Device scratch a launch needs (0 for most plans).  A runtime hosts it as a
 * private logical buffer of the step, as the reference does for cuBLASLt
 * workspaces (lib/Runtime/CUDA.cpp:759-764), so its plan verifier sees it.
 */
ASK_B200_API int ask_b200_plan_scratch_bytes(const ask_b200_plan *plan, size_t *bytes);

/*
 * Artifact-style JSON description of the plan: family, selected kernel and
 * strategy, grid/block, scratch, kernels per launch and the port map with
 * element types, element counts and index maps (the fields of the reference's
 * cuda_artifact, lib/Lowering/CUDA.cpp:396-407).  Writes at most `cap` bytes
 * including the terminating NUL; *needed receives the full size.
 */
ASK_B200_API int ask_b200_plan_describe(const ask_b200_plan *plan, char *buf, size_t cap, size_t *needed);

/* Kernels one ask_b200_plan_launch enqueues (for launch accounting). */
ASK_B200_API int ask_b200_plan_kernel_launches(const ask_b200_plan *plan, int *launches);

/*
 * Enqueue the step.  `ports` holds n_inputs + n_outputs device addresses,
 * inputs first (the reference's kernel parameter order, CUDA.cpp:177-208).
 * `scratch` is a device address of at least ask_b200_plan_scratch_bytes bytes
 * (ignored when that is 0).  `stream` is a cudaStream_t (NULL = legacy default).
 * Replaces launchKernel / launchPreCopyKernel (lib/Runtime/CUDA.cpp:360-371):
 * a scatter_add step's pre_copy (base -> output) is part of this launch.
 */
ASK_B200_API int ask_b200_plan_launch(const ask_b200_plan *plan, const uint64_t *ports, size_t n_ports, uint64_t scratch,
                         void *stream);

/*
 * Launch a reduce plan without any allocation by the caller or the library.
 * This entry point has no counterpart in the reference.  It exists for callers
 * that cannot call cudaMalloc when they launch: runtimes whose device memory is
 * wholly planned ahead by a pool (nothing may be added at launch time), and
 * hosts with a fixed device-memory budget, where cudaMalloc may fail or stall
 * the launching thread while the device synchronises.  A split
 * reduction's scratch (one partial record per CTA), or the chunk records of a
 * column reduction whose extent is split into chunks, then comes from a
 * file-scope device array of ASK_B200_NOALLOC_SCRATCH_BYTES (1 MiB) that every
 * GPU loading this library holds until the process exits; plans needing more
 * scratch than that (ask_b200_plan_scratch_bytes) are rejected with
 * ASK_B200_E_INVALID.
 * Only reduce plans are accepted (others: ASK_B200_E_UNSUPPORTED).  The first
 * call on a device looks up the array's address (cudaGetSymbolAddress) and
 * keeps it for the life of the process, keyed by device ordinal: the entry
 * point assumes one context per device (the runtime API's primary context) for
 * the whole process, so a caller that switches to another driver-API context,
 * or rebuilds the primary context after cudaDeviceReset, must not use it
 * afterwards.  Make that first call before any stream capture.  All calls share the array, which
 * keeps the last call's contents (the kernels overwrite every record they
 * read), so calls that overlap on the GPU race and must be serialised by the
 * caller.  Ports and stream are as for ask_b200_plan_launch.
 */
#define ASK_B200_NOALLOC_SCRATCH_BYTES (1u << 20)
ASK_B200_API int ask_b200_plan_launch_noalloc(const ask_b200_plan *plan, const uint64_t *ports, size_t n_ports,
                                              void *stream);

/*
 * Sharded plans.  A reduce plan whose outputs are 0-D may be split along its
 * leading axis across ranks (one process per GPU): every rank builds the plan
 * for its own slice with "index_base" set to the slice's global offset, and
 * ask_b200_plan_launch_sharded folds the slice into a partial record, exchanges
 * the records with one NCCL all-gather on `stream`, and combines them in rank
 * order, so every rank writes the same outputs.  The reference has no
 * multi-device path (each Session binds one device, lib/Runtime/CUDA.cpp:418-441);
 * these entry points are new.  NCCL is loaded at run time (libnccl.so.2).
 */
ASK_B200_API int ask_b200_comm_unique_id(unsigned char id[128]);
ASK_B200_API int ask_b200_comm_create(const unsigned char id[128], int nranks, int rank, int device, ask_b200_comm **out);
ASK_B200_API int ask_b200_comm_destroy(ask_b200_comm *comm);
ASK_B200_API int ask_b200_plan_launch_sharded(const ask_b200_plan *plan, ask_b200_comm *comm, const uint64_t *ports,
                                 size_t n_ports, uint64_t scratch, void *stream);
/*
 * The records cross GPUs by peer memory when every rank could map the others'
 * small exchange buffer (CUDA IPC over NVLink; decided once, at
 * ask_b200_comm_create, identically on every rank): one kernel stores this
 * rank's records into every rank's buffer, raises a flag per rank and waits
 * for every rank's flag -- a wait bounded by ASK_B200_EXCHANGE_TIMEOUT_MS
 * (default 1000 ms) -- then folds the records in rank order.  Otherwise the
 * NCCL all-gather runs.  Every rank must make the same sequence of sharded
 * launches, in one stream order per communicator (as for NCCL collectives):
 * two sharded launches of one communicator running at once on different
 * streams would take their epochs in different orders on different ranks.
 * The epoch lives on the device, so a captured CUDA graph of sharded
 * launches can be replayed.  ask_b200_comm_status reports whether the peer exchange is in use
 * and, synchronously, whether any wait ran out (ASK_B200_E_TIMEOUT: the
 * outputs of that launch were left unwritten and the communicator must be
 * destroyed; its exchange buffer then stays allocated until the process exits,
 * since a late peer may still store into it).  ask_b200_comm_destroy waits for
 * this device's work first.  No counterpart in the reference.
 */
ASK_B200_API int ask_b200_comm_status(ask_b200_comm *comm, int *status, int *peer_exchange);

/*
 * Seeded synthetic inputs (Philox4x32-10), generated on the device: element i
 * of stream `stream_id` is a pure function of (seed, stream_id, offset + i).
 * kind: 0 uniform f32 in [p0, p1); 1 normal f32 (mean p0, std p1); 2 normal f16;
 * 3 normal bf16; 4 raw i32; 5 Zipf(s = p0) i64 over ranks [0, p1); 6 the same as i32.
 * No reference counterpart: the reference holds no input generator.
 */
ASK_B200_API int ask_b200_generate(int kind, uint64_t seed, uint32_t stream_id, uint64_t offset, uint64_t count, double p0,
                      double p1, uint64_t dst, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ASK_B200_H */
