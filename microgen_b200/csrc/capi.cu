// C-ABI plumbing: status strings, error words, version, TMA descriptors.
#include <cstdlib>
#include <mutex>

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

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t get_encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(p);
  });
  return fn;
}

int mg_make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  PFN_encodeTiled_t enc = get_encode_fn();
  if (!enc) return MG_ERR_CUDA;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MG_OK : MG_ERR_INVALID_ARG;
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
  MG_CUDA_TRY(cudaStreamSynchronize(s));
  if (vals[0] != MG_OK) {  // the common case (no error) costs one read and one synchronisation
    MG_CUDA_TRY(cudaMemcpyFromSymbolAsync(&vals[1], g_mg_dev_error_info, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
    MG_CUDA_TRY(cudaStreamSynchronize(s));
  }
  *code = vals[0];
  if (info) *info = vals[1];
  if (clear && vals[0] != MG_OK) {
    const int zero[2] = {0, 0};
    MG_CUDA_TRY(cudaMemcpyToSymbolAsync(g_mg_dev_error, &zero[0], sizeof(int), 0, cudaMemcpyHostToDevice, s));
    MG_CUDA_TRY(cudaMemcpyToSymbolAsync(g_mg_dev_error_info, &zero[1], sizeof(int), 0, cudaMemcpyHostToDevice, s));
    MG_CUDA_TRY(cudaStreamSynchronize(s));
  }
  return MG_OK;
}
