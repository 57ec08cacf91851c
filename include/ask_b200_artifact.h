/*
 * ask_b200_artifact.h -- kernel artifacts for ASK's external-worker path.
 *
 * ASK loads external kernels as "external-kernel-artifact v2" documents
 * (schemas/external-kernel-artifact-v2.schema.json; docs/en/compilers.md,
 * "Minimal Response"): a cubin or PTX payload, one entry point whose
 * parameters are device pointers bound to ports and scalars, a fixed launch
 * and the element types to check.  Session::load (include/ask/Runtime/CUDA.h:75-78,
 * lib/Runtime/CUDA.cpp:499-541) checks the entry's parameter layout against
 * `parameterWidths` (0 = device pointer, 1/2/4/8 = scalar bytes).
 *
 * ask_b200_artifact_source turns one recipe step into the CUDA source of such
 * an entry for sm_100a; ask_b200/worker.py wraps it in ASK's worker process
 * interface (`--probe`, `--request R --output A`), compiles it and writes the
 * artifact.  ask_b200_runtime.h's ask_b200_kernel_load is the matching loader.
 */
#ifndef ASK_B200_ARTIFACT_H
#define ASK_B200_ARTIFACT_H

#include "ask_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * recipe_json: a step recipe (ask_b200.h).  options_json:
 *   {"entry": "name",
 *    "grid": [x, 1, 1],                 -- the launch grid the caller fixes
 *    "parameters": ["input:0", "output:0", "i32", ...]}
 * Each parameter is a port ("input:N" / "output:N", every port exactly once) or
 * a scalar ABI type (i1 i8 i16 i32 i64 u8 u16 u32 u64 fp16 bf16 fp32 fp64),
 * which the kernel accepts and ignores (every size is compiled in).
 * Result: {"entry", "body", "launch": {"grid", "block", "shared_bytes"},
 *          "parameter_widths": [...], "required_element_types": [...],
 *          "port_map": [...], "source": "<CUDA C++>"}.
 * Elementwise, reduce and gather steps are supported; scatter_add (which needs
 * the Runtime's pre_copy) and the fused softmax return ASK_B200_E_UNSUPPORTED.
 */
ASK_B200_API int ask_b200_artifact_source(const char *recipe_json, const char *options_json, char *buf, size_t cap,
                                          size_t *needed);

#ifdef __cplusplus
}
#endif

#endif /* ASK_B200_ARTIFACT_H */
