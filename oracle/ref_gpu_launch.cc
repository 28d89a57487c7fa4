// Launcher of the reference's GPU SHA-256 kernel. TEST/BENCH INFRASTRUCTURE ONLY.
//
// Loads the PTX that oracle/ref_gpu_build.py produced from the reference's own
// kernel text (core/common/artifact_hash_gpu.cc:193-412, NVRTC, compute_100) into
// the device's primary context -- the driver JIT-compiles it for the GPU, as the
// reference's cuModuleLoadDataEx does -- and launches it with the reference's
// configuration (artifact_hash_gpu.cc:771-781): 512 threads per block, grid
// min(ceil(leaves / 512), 8 * SM count), arguments (base, chunk stride, total
// size, digests, leaf count). Used only by bench.py to time the reference kernel
// beside the product kernel on the same bytes; the product never links it.
#include <cuda.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

CUmodule g_module = nullptr;
CUfunction g_kernel = nullptr;
int g_sms = 0;
std::string g_error;

int fail(const char* what, CUresult r) {
  const char* s = nullptr;
  cuGetErrorString(r, &s);
  g_error = std::string(what) + ": " + (s ? s : "unknown CUDA driver error");
  return static_cast<int>(r);
}

}  // namespace

extern "C" const char* ref_gpu_last_error(void) { return g_error.c_str(); }

// Loads the reference kernel on `device` (its primary context, shared with the CUDA
// runtime). Returns 0 or a CUresult.
extern "C" int ref_gpu_load(const char* ptx_path, int device) {
  FILE* f = std::fopen(ptx_path, "rb");
  if (f == nullptr) {
    g_error = std::string("cannot open ") + ptx_path;
    return -1;
  }
  std::vector<char> ptx;
  char buf[1 << 16];
  size_t got;
  while ((got = std::fread(buf, 1, sizeof buf, f)) > 0) ptx.insert(ptx.end(), buf, buf + got);
  std::fclose(f);
  ptx.push_back('\0');
  CUresult r = cuInit(0);
  if (r != CUDA_SUCCESS) return fail("cuInit", r);
  CUdevice dev;
  if ((r = cuDeviceGet(&dev, device)) != CUDA_SUCCESS) return fail("cuDeviceGet", r);
  CUcontext ctx;
  if ((r = cuDevicePrimaryCtxRetain(&ctx, dev)) != CUDA_SUCCESS) return fail("cuDevicePrimaryCtxRetain", r);
  if ((r = cuCtxSetCurrent(ctx)) != CUDA_SUCCESS) return fail("cuCtxSetCurrent", r);
  if ((r = cuDeviceGetAttribute(&g_sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev)) != CUDA_SUCCESS)
    return fail("cuDeviceGetAttribute", r);
  if ((r = cuModuleLoadData(&g_module, ptx.data())) != CUDA_SUCCESS) return fail("cuModuleLoadData", r);
  if ((r = cuModuleGetFunction(&g_kernel, g_module, "tensorcast_sha256_leaf_kernel")) != CUDA_SUCCESS)
    return fail("cuModuleGetFunction", r);
  return 0;
}

// One launch of the reference kernel over [d_src, d_src + total): leaf i of
// `leaf` bytes gets its digest at d_digests + 32*i. Stream-ordered.
extern "C" int ref_gpu_sha256_leaves(const void* d_src, uint64_t total, uint64_t leaf, void* d_digests,
                                     uint32_t n_leaves, void* stream) {
  if (g_kernel == nullptr) {
    g_error = "ref_gpu_load was not called";
    return -1;
  }
  CUdeviceptr base = reinterpret_cast<CUdeviceptr>(d_src);
  CUdeviceptr digests = reinterpret_cast<CUdeviceptr>(d_digests);
  unsigned long long stride = leaf, size = total;  // the kernel's uint64_t is unsigned long long
  unsigned int count = n_leaves;
  void* params[] = {&base, &stride, &size, &digests, &count};
  const unsigned int threads = 512;
  const unsigned int blocks = (count + threads - 1) / threads;
  const unsigned int max_grid = g_sms > 0 ? static_cast<unsigned int>(g_sms) * 8u : 1u;
  const unsigned int grid = blocks == 0 ? 1u : (blocks < max_grid ? blocks : max_grid);
  CUresult r = cuLaunchKernel(g_kernel, grid, 1, 1, threads, 1, 1, 0, static_cast<CUstream>(stream), params, nullptr);
  if (r != CUDA_SUCCESS) return fail("cuLaunchKernel(tensorcast_sha256_leaf_kernel)", r);
  return 0;
}
