// Fixed-scratch launch: ask_b200_plan_launch_noalloc.
//
// Some callers cannot call cudaMalloc when they launch a step: runtimes whose
// device memory is entirely planned ahead by a pool (ASK's Runtime sizes and
// verifies every buffer when a plan is prepared, so a launch has no way to add
// one), and embedded or real-time hosts with a fixed device-memory budget, for
// which cudaMalloc may fail or stall the launching thread while the device
// synchronises.  For the reductions that need scratch memory -- the split
// reduction, which keeps one partial record per CTA between its two kernels,
// and the column reduction whose extent is split into chunks, which keeps one
// record per chunk and column -- this entry point supplies that scratch from a
// file-scope device array instead, so the caller passes only inputs and
// outputs and nothing is allocated.
//
// The array is kFixedScratchBytes (1 MiB) on every GPU that loads this library
// and stays allocated until the process exits.  Its address is looked up once
// per device with cudaGetSymbolAddress the first time the entry point runs on
// that device; that first call should therefore happen before any stream
// capture.  The address is kept by device ordinal for the life of the process,
// which assumes one context per device (the runtime API's primary context):
// after a switch to another driver-API context, or a primary context rebuilt by
// cudaDeviceReset, the kept address would belong to the old context.
// Every call shares the array and it keeps the previous call's contents: both
// reductions write every record they later read, so nothing needs clearing,
// but calls that overlap on the GPU (different streams, or the same plan
// launched concurrently) race on the array and must be serialised by the
// caller.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/ask_b200.h"

extern "C" int askb_internal_launch_reduce_fixed_scratch(const ask_b200_plan* plan, const uint64_t* ports,
                                                         size_t n_ports, void* scratch, size_t capacity,
                                                         void* stream);
extern "C" void askb_internal_set_error(const char* message);

namespace {

constexpr size_t kFixedScratchBytes = ASK_B200_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_fixed_scratch[kFixedScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

}  // namespace

extern "C" int ask_b200_plan_launch_noalloc(const ask_b200_plan* plan, const uint64_t* ports, size_t n_ports,
                                            void* stream) {
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    askb_internal_set_error((std::string("cudaGetDevice: ") + cudaGetErrorString(err)).c_str());
    return ASK_B200_E_CUDA;
  }
  if (device < 0 || device >= kMaxDevices) {
    askb_internal_set_error("device ordinal out of range for the fixed scratch array");
    return ASK_B200_E_DEVICE;
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[device]) {
      // Host code names the array only to look up its device address; the
      // symbol itself is a host-side stand-in and must never reach a kernel.
      void* address = nullptr;
      err = cudaGetSymbolAddress(&address, g_fixed_scratch);
      if (err != cudaSuccess || !address) {
        askb_internal_set_error((std::string("cudaGetSymbolAddress(fixed scratch): ") +
                                 cudaGetErrorString(err)).c_str());
        return ASK_B200_E_CUDA;
      }
      g_scratch_address[device] = address;
    }
    scratch = g_scratch_address[device];
  }
  return askb_internal_launch_reduce_fixed_scratch(plan, ports, n_ports, scratch, kFixedScratchBytes, stream);
}
