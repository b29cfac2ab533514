// Host-side helpers shared by the launchers: thread-local error text and kernel launch with
// optional programmatic dependent launch (PDL).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace aipu {

// status codes returned by every C entry point (mirrored in include/aipu_q4k.h)
enum : int { OK = 0, EINVAL_ = -1, ECUDA_ = -2, ETIMEOUT_ = -3, ENCCL_ = -4, ENOMEM_ = -5 };

int set_error(int code, const char* msg);
int set_cuda_error(cudaError_t e, const char* where);
const char* last_error();

// Launch `kern` with the given configuration. When `pdl` is true the launch carries
// cudaLaunchAttributeProgrammaticStreamSerialization, so it may start while the previous kernel on
// the stream drains; kernels call griddepcontrol.wait before touching inputs that the previous
// kernel produces.
int launch_kernel(const void* kern, dim3 grid, dim3 block, int smem, cudaStream_t stream, bool pdl, void* arg0);

int num_sms_of_current_device();

// Raise a kernel's dynamic shared-memory limit once per device (the attribute is per device, so a
// process with contexts on several devices sets it on each). `done` is the caller's per-kernel
// table of 64 device flags.
int set_smem_attr_once(const void* kern, int bytes, bool* done, const char* what);

// Encode a tiled TMA tensor map (no swizzle, no interleave, OOB reads return 0). The driver entry
// point is looked up through the runtime, so the library does not link libcuda.
// dims/box in elements (innermost first); strides in bytes for dims 1..rank-1.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides, const cuuint32_t* box);

}  // namespace aipu
