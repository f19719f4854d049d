// Host-side runtime shared by every C-ABI entry point: status codes, the
// thread-local error string, the per-device status word that bounded device
// waits report into, and TMA tensor-map encoding through the driver entry
// point (so the library links only the static CUDA runtime and still loads on
// a machine without a GPU driver).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <string>

#include "../../include/neso_b200.h"
#include "common.cuh"

namespace neso {

// Record an error message for neso_last_error_string() and return `code`.
int fail(int code, const char* fmt, ...);
// Clear the thread's error string and return NESO_OK.
int ok();

// Map a CUDA runtime error to NESO_ERR_LAUNCH with a message.
int cuda_fail(cudaError_t e, const char* what);

// Device status block for the device that owns `stream` (lazily allocated
// once per device, 4 ints: code, where, block, thread).
int device_status(DevStatus* out);

// Scratch buffer of at least `bytes` for work queued on `stream` (one buffer
// per device, stream and kind, grown on demand; growing synchronises the
// stream first). Stays allocated until the process exits. Two kinds, so one
// call can hold both: split-K partial sums, and inputs converted to the
// layout a kernel reads (fp32 -> fp16 attention operands, int32-held int8
// weights -> int8).
constexpr int kWorkspacePartials = 0;
constexpr int kWorkspaceInputs = 1;
int stream_workspace(cudaStream_t stream, size_t bytes, void** out, int which = kWorkspacePartials);
// kStreamCounters zero-initialised ints for kernels queued on `stream` that
// hand out or count work through atomics (one block per device and stream,
// allocated and zeroed on first use). A kernel that uses them leaves them
// zero on exit. Slots: [0, 2) the FA2 persistent kernel's unit tickets,
// [kGemvCounterBase, kGemvCounterEnd) the small-M GEMV's channel blocks,
// [kGemmCounterBase, kStreamCounters) the GEMM's K-split tail tiles.
constexpr int kStreamCounters = 4096;
constexpr int kGemvCounterBase = 64;
constexpr int kGemvCounterEnd = 1024;
constexpr int kGemmCounterBase = 2048;
int stream_counters(cudaStream_t stream, int** out);

// Opt a kernel into `smem_bytes` of dynamic shared memory and return its
// attributes; done once per (device, kernel) and cached, so per-call launches
// do not pay for the attribute calls.
int kernel_setup(const void* kern, int smem_bytes, cudaFuncAttributes* attrs);

// Number of SMs on the current device (cached per device).
int sm_count();

// Encode a tiled tensor map (fp16/int8/...) with 128-byte swizzle and zero OOB
// fill. dims/strides follow the driver convention (dims[0] innermost; strides
// are byte strides of dims 1..rank-1).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* gaddr, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline cudaStream_t as_stream(neso_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Launch with programmatic stream serialization (programmatic dependent
// launch): the kernel's CTAs may be scheduled, into SM slots the previous
// kernel on the stream no longer uses, before that kernel has finished, so
// its launch and prologue overlap the previous kernel's tail. The kernel must
// call pdl_wait() before it reads or writes global memory that an earlier
// kernel on the stream may touch; launched without the attribute, pdl_wait()
// returns at once.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace neso
