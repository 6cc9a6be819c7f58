// TEST INFRASTRUCTURE ONLY -- driver API stand-ins for the host-only build of the
// reference gather (oracle/_ref/libgfd_ref_cpu.so).  That build only runs
// CpuPollingThread::parallel_gather, which calls none of these; they exist so the
// reference objects link on a machine without libcuda.  Each reports "no device".
#include <cuda.h>

extern "C" {
CUresult cuCtxGetCurrent(CUcontext* c) { if (c) *c = nullptr; return CUDA_ERROR_NO_DEVICE; }
CUresult cuCtxGetStreamPriorityRange(int*, int*) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuCtxPopCurrent_v2(CUcontext*) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuCtxPushCurrent_v2(CUcontext) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuEventCreate(CUevent*, unsigned int) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuEventDestroy_v2(CUevent) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuEventQuery(CUevent) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuEventRecord(CUevent, CUstream) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuEventSynchronize(CUevent) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuGetErrorString(CUresult, const char** s) { if (s) *s = "no device"; return CUDA_SUCCESS; }
CUresult cuMemcpyHtoDAsync_v2(CUdeviceptr, const void*, size_t, CUstream) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuStreamCreate(CUstream*, unsigned int) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuStreamCreateWithPriority(CUstream*, unsigned int, int) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuStreamDestroy_v2(CUstream) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuStreamSynchronize(CUstream) { return CUDA_ERROR_NO_DEVICE; }
CUresult cuStreamWaitEvent(CUstream, CUevent, unsigned int) { return CUDA_ERROR_NO_DEVICE; }
}
