/*
 * ask_b200_runtime.h -- the runtime layer that hosts ask_b200 plans as the
 * steps of an execution plan: sessions, device buffers, prepared programs and
 * completion events.  It mirrors the reference Runtime's C++ surface
 * (include/ask/Runtime/CUDA.h:66-175; lib/Runtime/CUDA.cpp:418-1005).  A step
 * is either an ask_b200 plan (a "recipe step") whose ports are bound to
 * logical buffers of the program, or a loaded kernel (Session::load, e.g. a
 * kernel artifact from ask_b200_artifact.h) with its arguments and launch.
 *
 *   Session            one device, one non-blocking stream, usage counters
 *                      (Session::create / allocate / importBuffer /
 *                      prepareProgram / synchronize / reap / stats)
 *   DeviceBuffer       device memory owned by the session or imported
 *   PreparedProgram    buffer sizes, public inputs/outputs and steps, verified
 *                      once (the reference's PASS plan check,
 *                      lib/Pass/Pass.cpp:12-208) with internal buffers mapped
 *                      to reusable workspace slots; submit() binds the public
 *                      ports, run() also allocates the outputs
 *   Kernel             a loaded cubin/PTX entry whose parameter layout was
 *                      checked against declared widths (Session::load)
 *   Event              completion of one submission; it keeps the submission's
 *                      buffers and workspace alive until the GPU is done
 *
 * Graph mode (graph = 1) records each step as a child graph of one CUDA graph
 * per workspace, with the plan's data dependencies as edges, and replays it;
 * later submissions whose public addresses changed re-record only the steps
 * bound to those ports (cudaGraphExecChildGraphNodeSetParams).
 *
 * A program is JSON:
 *   {"buffer_sizes": [bytes, ...], "inputs": [buffer, ...], "outputs": [buffer, ...],
 *    "steps": [{"recipe": "<ask_b200 recipe JSON text>", "inputs": [buffer, ...],
 *               "outputs": [buffer, ...], "pre_copy": {"source": b, "destination": b}}]}
 * A step's inputs and outputs bind the recipe's ports in port-map order; each
 * bound buffer's size must equal the port's bytes.  A plan that needs scratch
 * gets a private logical buffer, as the reference does for a cuBLASLt
 * workspace (lib/Runtime/CUDA.cpp:759-764).  "pre_copy" is the reference's
 * PlanStep::preCopy (include/ask/Runtime/CUDA.h:50-62): a device-to-device
 * copy enqueued before the step.  A scatter_add recipe already performs its own
 * pre-copy (out = base) inside its launch and needs none.
 *
 * A kernel step (ask_b200_program_prepare_kernels) replaces "recipe" with
 *   "kernel": k (index into the kernels passed), "grid": [x, y, z],
 *   "block": [x, y, z], "shared_bytes": n,
 *   "arguments": [{"buffer": b, "align": a} | {"buffer": -1} | {"scalar": "<hex ABI bytes>"}, ...]
 * with one argument per kernel parameter: pointer parameters bind step ports
 * (every port exactly once) or null, scalar parameters carry exactly their
 * width in little-endian bytes (the reference's PlanArgument).  The optional
 * "align" is the address alignment the kernel needs for that pointer (its
 * element size): a submission binding a public buffer at another address is
 * refused before anything is enqueued.
 *
 * All entry points return 0 or a negative ASK_B200_E_* status with the
 * message in ask_b200_last_error() (ask_b200.h).  Handles are reference
 * counted: *_release drops the caller's handle, and an object lives on while
 * another object (an event, a program, a buffer) still needs it.
 */
#ifndef ASK_B200_RUNTIME_H
#define ASK_B200_RUNTIME_H

#include "ask_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ask_b200_session ask_b200_session;
typedef struct ask_b200_buffer ask_b200_buffer;
typedef struct ask_b200_program ask_b200_program;
typedef struct ask_b200_event ask_b200_event;
typedef struct ask_b200_kernel ask_b200_kernel;

/* One argument of Session::submit: a buffer (NULL for a null pointer) for a
 * pointer parameter, or scalar_bytes bytes at scalar for a scalar one.  align
 * (0 or 1 = none) is the address alignment the kernel needs for a pointer --
 * its element size; a buffer at another address is refused before launch. */
typedef struct ask_b200_kernel_arg {
  ask_b200_buffer *buffer;
  const void *scalar;
  size_t scalar_bytes;
  size_t align;
} ask_b200_kernel_arg;

/* Session::create(device) (lib/Runtime/CUDA.cpp:418-441). */
ASK_B200_API int ask_b200_session_create(int device, ask_b200_session **out);
/* Session::close + drop the handle: waits for pending submissions first. */
ASK_B200_API int ask_b200_session_release(ask_b200_session *session);
ASK_B200_API int ask_b200_session_synchronize(ask_b200_session *session);
/* Session::reap: retire completed submissions (their workspaces become idle). */
ASK_B200_API int ask_b200_session_reap(ask_b200_session *session);
/* The session's cudaStream_t (Session::stream). */
ASK_B200_API int ask_b200_session_stream(ask_b200_session *session, void **stream);
/* Session::waitForExternalStream: later work waits for `stream`'s current tail. */
ASK_B200_API int ask_b200_session_wait_stream(ask_b200_session *session, void *stream);
/* Session::stats as a JSON object of counters (written as ask_b200_plan_describe). */
ASK_B200_API int ask_b200_session_stats(ask_b200_session *session, char *buf, size_t cap, size_t *needed);

/* Session::allocate / importBuffer, DeviceBuffer::pointer/size/readonly/copy*. */
ASK_B200_API int ask_b200_buffer_allocate(ask_b200_session *session, size_t bytes, ask_b200_buffer **out);
ASK_B200_API int ask_b200_buffer_import(ask_b200_session *session, uint64_t pointer, size_t bytes, int readonly,
                                        ask_b200_buffer **out);
ASK_B200_API int ask_b200_buffer_info(const ask_b200_buffer *buffer, uint64_t *pointer, size_t *bytes, int *readonly);
ASK_B200_API int ask_b200_buffer_copy_from_host(ask_b200_buffer *buffer, const void *src, size_t bytes);
ASK_B200_API int ask_b200_buffer_copy_to_host(const ask_b200_buffer *buffer, void *dst, size_t bytes);
ASK_B200_API int ask_b200_buffer_release(ask_b200_buffer *buffer);

/* Session::prepareProgram(sizes, inputs, outputs, steps, graph). */
ASK_B200_API int ask_b200_program_prepare(ask_b200_session *session, const char *program_json, int graph,
                                          ask_b200_program **out);
/* JSON: slots and capacities, buffer-to-slot assignments, dependencies, step kernels. */
ASK_B200_API int ask_b200_program_describe(const ask_b200_program *program, char *buf, size_t cap, size_t *needed);
/* PreparedProgram::submit(inputs, outputs). */
ASK_B200_API int ask_b200_program_submit(ask_b200_program *program, ask_b200_buffer *const *inputs, size_t n_inputs,
                                         ask_b200_buffer *const *outputs, size_t n_outputs, ask_b200_event **event);
/* PreparedProgram::run(inputs): outputs[] receives new handles (an output
 * that is a program input is that input's buffer). */
ASK_B200_API int ask_b200_program_run(ask_b200_program *program, ask_b200_buffer *const *inputs, size_t n_inputs,
                                      ask_b200_buffer **outputs, size_t n_outputs, ask_b200_event **event);
ASK_B200_API int ask_b200_program_release(ask_b200_program *program);

/* Session::prepareProgram with kernel steps: "kernel": k in a step indexes kernels[]. */
ASK_B200_API int ask_b200_program_prepare_kernels(ask_b200_session *session, const char *program_json,
                                                  ask_b200_kernel *const *kernels, size_t n_kernels, int graph,
                                                  ask_b200_program **out);

/*
 * Session::load(image, entry, requiredTypes, arch, parameterWidths)
 * (lib/Runtime/CUDA.cpp:499-541): a cubin ELF image for compute capability
 * arch/10.arch%10 (or PTX text for at least arch), the entry's parameter widths
 * (0 = device pointer, 1/2/4/8 = scalar bytes) checked against its layout,
 * and the element types the session must support.  Loaded once per
 * (image, entry) per session; a second load returns the cached kernel.
 */
ASK_B200_API int ask_b200_kernel_load(ask_b200_session *session, const void *image, size_t bytes, const char *entry,
                                      const char *const *required_types, size_t n_types, int arch,
                                      const unsigned *widths, size_t n_widths, ask_b200_kernel **out);
/* Kernel::entry / Kernel::maxThreads. */
ASK_B200_API int ask_b200_kernel_info(const ask_b200_kernel *kernel, char *entry, size_t cap, size_t *needed,
                                      unsigned *max_threads);
ASK_B200_API int ask_b200_kernel_release(ask_b200_kernel *kernel);
/* Session::submit(kernel, arguments, grid, block, sharedBytes) (lib/Runtime/CUDA.cpp:568-600). */
ASK_B200_API int ask_b200_kernel_submit(ask_b200_session *session, ask_b200_kernel *kernel,
                                        const ask_b200_kernel_arg *args, size_t n_args, const unsigned grid[3],
                                        const unsigned block[3], unsigned shared_bytes, ask_b200_event **event);

/* Event::query / Event::wait. */
ASK_B200_API int ask_b200_event_query(ask_b200_event *event, int *done);
ASK_B200_API int ask_b200_event_wait(ask_b200_event *event);
ASK_B200_API int ask_b200_event_release(ask_b200_event *event);

/*
 * The plan verifier on its own (pass::checkAllocationPlan,
 * lib/Pass/Pass.h:50-53), host only.  JSON:
 *   {"buffer_count": n, "public_inputs": [...], "public_outputs": [...],
 *    "steps": [{"inputs": [...], "outputs": [...]}], "buffer_sizes": [...],
 *    "assignments": [[buffer, slot], ...], "slot_capacity_bytes": [...],
 *    "graph": false, "dependencies": [[...], ...]}
 * *pass is 1 or 0; buf receives the explanation ("" on pass).  Omitting
 * "buffer_sizes" checks the plan alone (pass::checkPlan).
 */
ASK_B200_API int ask_b200_allocation_check(const char *allocation_json, int *pass, char *buf, size_t cap,
                                           size_t *needed);
/*
 * The slot assigners on their own, host only: from the plan fields above plus
 * "buffer_sizes", write {"assignments": ..., "slot_capacity_bytes": ...,
 * "dependencies": ...} for stream order (graph = 0) or graph order (graph = 1).
 */
ASK_B200_API int ask_b200_allocation_assign(const char *plan_json, int graph, char *buf, size_t cap, size_t *needed);

#ifdef __cplusplus
}
#endif

#endif /* ASK_B200_RUNTIME_H */
