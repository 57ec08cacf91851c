/*
 * ask_b200_lower.h -- lowering adapter from ASK step sources to ask_b200
 * recipes, the replacement for ask::lowerToCUDALLVM on sm_100
 * (lib/Lowering/CUDA.cpp:152-419, reached through codegen(..., {CUDALLVM, 100})
 * or `ask-opt --emit-cuda-llvm --cuda-arch 100`, tools/ask-opt.cpp:115-133).
 *
 * Input is what the reference's partitioner emits (lib/Frontend/Partition.cpp):
 * each owned step's module printed as MLIR text ("step_sources") and the
 * execution plan that binds steps to buffers.  The supported subset is the hot
 * path: elementwise ops over the step's iteration shape, whose arguments may
 * be read through broadcast_in_dim, transpose, slice, pad, reshape and
 * concatenate (as strided, windowed views of the argument) and iota -- a
 * reshape of a transposed, sliced or padded value, which no strided window
 * expresses, is read at the same row-major position through a second,
 * inner window (one such reshape per operand);
 * reductions (sum, prod, max, min, any, all, argmax, argmin) over any set
 * of axes (a scattered set is gathered last by a transpose), their operands
 * built the same way; gather and
 * scatter_add.  Steps outside it fail
 * with ASK_B200_E_UNSUPPORTED and a message naming the op (matmul steps, two
 * such reshapes stacked on one operand); index maps of computed elementwise
 * values move onto their operands, pads and concatenates of them become
 * coordinate selects.
 */
#ifndef ASK_B200_LOWER_H
#define ASK_B200_LOWER_H

#include "ask_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * One step source (a module holding one func.func of ASK ops) to
 * {"recipe": {...}, "input_arguments": [k, ...], "cuda_lowering": {...}}:
 * recipe input port i reads the function's argument input_arguments[i];
 * outputs follow the function's return order.  "cuda_lowering" carries the
 * diagnostics fields of the reference's CUDA lowering report
 * (lib/Lowering/CUDA.cpp:408-417: statistics_stage, kernel_count, indexing,
 * warp_reduction_groups, output_loop_count, input_load_count,
 * reduction_loop_count, zero_element_outputs, temporary_buffer_count, groups,
 * bool_storage, cast_semantics and, for scatter_add, pre_copy {input:
 * argument of the base, output}) for the kernels this library launches, plus
 * "kernel", "strategy" and "scratch_bytes".  Text is written as by
 * ask_b200_plan_describe.
 */
ASK_B200_API int ask_b200_lower_step(const char *step_source, char *buf, size_t cap, size_t *needed);

/*
 * A partition report ({"execution_plan": {...}, "step_sources": {...}}, the
 * reference's report fields) to a runtime program for
 * ask_b200_program_prepare (ask_b200_runtime.h): buffer sizes from the plan's
 * buffer shapes and element types, public inputs and outputs, and one recipe
 * step per owned step with its ports bound to the plan's buffers.  A step
 * whose results one recipe cannot hold (elementwise results of different
 * shapes, reductions over different axes or operand shapes) becomes one
 * program step per group of results, ids "<step>#<k>", each writing its own
 * outputs -- the reference's one batch per output shape
 * (lib/Lowering/CUDA.cpp:210-244).  A gather or scatter_add whose operands
 * are computed in the step reads them from internal buffers (appended after
 * the plan's buffers) that elementwise steps write first.  Each recipe step
 * carries its "cuda_lowering" report.  External and library steps keep their
 * place and buffers as {"id", "unresolved": {"kind", "function",
 * "external_id" | "library"}, "inputs", "outputs"}, listed again in
 * "unresolved_steps": the caller replaces "unresolved" with a loaded kernel
 * ("kernel", "grid", "block", "arguments"; ask_b200_program_prepare_kernels)
 * before preparing the program.
 * ask_b200_lower_step returns one recipe and rejects both kinds of step.
 */
ASK_B200_API int ask_b200_lower_report(const char *report_json, char *buf, size_t cap, size_t *needed);

#ifdef __cplusplus
}
#endif

#endif /* ASK_B200_LOWER_H */
