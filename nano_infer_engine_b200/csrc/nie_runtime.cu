// Host-side runtime of the library: per-thread error messages, cached device
// properties, peer access and the tensor-map encoder (resolved through the
// runtime's driver entry point so the library needs no -lcuda at link time).
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "nie_common.cuh"

namespace nie {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NIE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return NIE_OK;
}

static std::mutex g_mu;
static int g_sm_count[64] = {0};

int sm_count(int device) {
  if (device < 0 || device >= 64) return -1;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sm_count[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
    g_sm_count[device] = v;
  }
  return g_sm_count[device];
}

// Raise `kernel`'s dynamic shared memory limit on the current device to at
// least `bytes`, per (device, slot): function attributes belong to the
// device's context, so a thread that drives two GPUs must set them on each.
static size_t g_smem_opt_in[64][kSmemSlots];

int opt_in_smem(int slot, const void* kernel, size_t bytes) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || slot < 0 || slot >= kSmemSlots)
    return fail(NIE_ERR_CUDA, "cannot resolve the current device for a shared-memory opt-in");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_smem_opt_in[dev][slot] < bytes) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return fail(NIE_ERR_CUDA, "shared memory opt-in of %zu bytes: %s", bytes, cudaGetErrorString(e));
    g_smem_opt_in[dev][slot] = bytes;
  }
  return NIE_OK;
}

// Device whose SMs a launch on `stream` uses.  A kernel launch requires the
// stream to belong to the current device, so the current device is the
// answer; querying the stream itself (cudaStreamGetDevice) would invalidate a
// CUDA-graph capture in progress on it.
int stream_device(cudaStream_t stream) {
  (void)stream;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, uint32_t rank, void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return fail(NIE_ERR_CUDA, "cannot resolve cuTensorMapEncodeTiled");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  uint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dt, rank, base, dims, strides_bytes, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NIE_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return NIE_OK;
}

}  // namespace nie

extern "C" int nie_version(void) { return 100; }

extern "C" const char* nie_last_error(void) { return nie::g_last_error; }

extern "C" int nie_device_sm_count(int device) { return nie::sm_count(device); }

namespace nie {
static PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;
}

extern "C" int nie_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  NIE_REQUIRE(ptr && handle_out && offset_out, "null pointer argument");
  {
    std::lock_guard<std::mutex> lk(nie::g_mu);
    if (nie::g_addr_range == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 3020, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return nie::fail(NIE_ERR_CUDA, "cannot resolve cuMemGetAddressRange");
      nie::g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
    }
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = nie::g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return nie::fail(NIE_ERR_CUDA, "cuMemGetAddressRange failed (CUresult %d)", (int)r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return nie::fail(NIE_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return NIE_OK;
}

extern "C" int nie_ipc_import(const void* handle, uint64_t offset, void** ptr_out, void** base_out) {
  NIE_REQUIRE(handle && ptr_out && base_out, "null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return nie::fail(NIE_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return NIE_OK;
}

extern "C" int nie_ipc_close(void* base) {
  NIE_REQUIRE(base, "null pointer argument");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return nie::fail(NIE_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return NIE_OK;
}

extern "C" int nie_enable_peer_access(int device, int peer_device) {
  if (device == peer_device) return NIE_OK;
  int can = 0;
  if (cudaDeviceCanAccessPeer(&can, device, peer_device) != cudaSuccess)
    return nie::fail(NIE_ERR_CUDA, "cudaDeviceCanAccessPeer(%d, %d) failed", device, peer_device);
  if (!can) return nie::fail(NIE_ERR_UNSUPPORTED, "device %d cannot access peer %d", device, peer_device);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    e = cudaSuccess;
  }
  if (prev >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess) return nie::fail(NIE_ERR_CUDA, "cudaDeviceEnablePeerAccess: %s", cudaGetErrorString(e));
  return NIE_OK;
}
