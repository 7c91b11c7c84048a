// C-ABI plumbing: status strings, error words, version.
#include <cstdlib>

#include "common.cuh"

__device__ int g_mg_dev_error = 0;
__device__ int g_mg_dev_error_info = 0;

static thread_local int t_last_cuda_error = 0;

bool mg_pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("MG_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int mg_set_cuda_error(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return MG_ERR_CUDA;
}

extern "C" int mg_abi_version(void) { return MG_ABI_VERSION; }

extern "C" const char* mg_status_string(int status) {
  switch (status) {
    case MG_OK: return "ok";
    case MG_ERR_INVALID_ARG: return "invalid argument";
    case MG_ERR_UNSUPPORTED: return "unsupported shape";
    case MG_ERR_CUDA: return "CUDA runtime error";
    case MG_ERR_TIMEOUT: return "bounded device wait timed out";
    case MG_ERR_DEVICE: return "device-side check failed";
    default: return "unknown status";
  }
}

extern "C" int mg_last_cuda_error(void) { return t_last_cuda_error; }

extern "C" int mg_device_error(void* stream, int clear, int* code, int* info) {
  if (!code) return MG_ERR_INVALID_ARG;
  cudaStream_t s = mg_stream(stream);
  int vals[2] = {0, 0};
  MG_CUDA_TRY(cudaMemcpyFromSymbolAsync(&vals[0], g_mg_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
  MG_CUDA_TRY(cudaMemcpyFromSymbolAsync(&vals[1], g_mg_dev_error_info, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
  MG_CUDA_TRY(cudaStreamSynchronize(s));
  *code = vals[0];
  if (info) *info = vals[1];
  if (clear) {
    const int zero[2] = {0, 0};
    MG_CUDA_TRY(cudaMemcpyToSymbolAsync(g_mg_dev_error, &zero[0], sizeof(int), 0, cudaMemcpyHostToDevice, s));
    MG_CUDA_TRY(cudaMemcpyToSymbolAsync(g_mg_dev_error_info, &zero[1], sizeof(int), 0, cudaMemcpyHostToDevice, s));
    MG_CUDA_TRY(cudaStreamSynchronize(s));
  }
  return MG_OK;
}
