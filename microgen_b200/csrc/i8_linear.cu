// INT8 weight-only linear y = epi(x · (q·s)ᵀ + b) for the decode path.
//
// Two kernels share one contract (include/microgen_b200.h):
//
// * i8_gemv_simt — CUDA cores. One warp per output row, 128-bit int8 loads, fp32
//   accumulation, the per-row scale applied once after the K reduction.
//
// * i8_gemm_tc   — tcgen05 tensor cores, "swap-AB": the weight rows are the MMA's
//   M=128 dimension and the tokens its N (= MP, the token count padded to 16..256),
//   so a decode batch of 1..256 tokens is one MMA tile per 128 weight rows.
//   Per 128-wide K block:
//     warp 4      TMA-loads the int8 weight tile [128 rows x 128 B] (128B-swizzled)
//                 and the activation tile [MP x 128] bf16 (two 64-wide swizzled boxes);
//     warps 0..3  (thread t <-> weight row t <-> TMEM lane t) convert the int8 row
//                 to bf16 (exact) and tcgen05.st it into a TMEM A buffer;
//     warp 5      issues 8 x tcgen05.mma kind::f16 (A from TMEM, B = activations
//                 from shared memory) accumulating fp32 into TMEM.
//   Split-K: the `split` CTAs of a thread-block cluster share one 128-row tile and
//   divide its K blocks; after the mainloop each CTA parks its fp32 accumulator in
//   shared memory and the cluster reduces it through distributed shared memory
//   (fixed order, deterministic), applying scale, bias and the epilogue.
#include <mutex>

#include "common.cuh"

namespace {

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float gelu_tanh_f(float v) {
  return 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

__device__ __forceinline__ void store_out(int epi, void* y, int64_t idx, float v) {
  switch (epi) {
    case MG_EPI_STORE_BF16: static_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v); break;
    case MG_EPI_STORE_F32: static_cast<float*>(y)[idx] = v; break;
    case MG_EPI_ADD_F32: static_cast<float*>(y)[idx] += v; break;
    case MG_EPI_GELU_BF16: static_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(gelu_tanh_f(v)); break;
    default: break;
  }
}

// Weight row of output feature f in the SwiGLU-interleaved layout: groups of 128 rows,
// 64 gate rows followed by the 64 matching up rows.
__device__ __forceinline__ int64_t swiglu_gate_row(int64_t f) { return (f >> 6) * 128 + (f & 63); }

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ------------------------------------------------------------------------------------------------
// CUDA-core GEMV
// ------------------------------------------------------------------------------------------------
constexpr int kSimtWarps = 8;
constexpr int kSimtMC = 4;  // token rows per pass

__device__ __forceinline__ float dot16(const float (&w)[16], const __nv_bfloat16* xp) {
  const uint4 a = *reinterpret_cast<const uint4*>(xp);
  const uint4 b = *reinterpret_cast<const uint4*>(xp + 8);
  float s = 0.f;
  s = fmaf(w[0], bf16lo(a.x), s);
  s = fmaf(w[1], bf16hi(a.x), s);
  s = fmaf(w[2], bf16lo(a.y), s);
  s = fmaf(w[3], bf16hi(a.y), s);
  s = fmaf(w[4], bf16lo(a.z), s);
  s = fmaf(w[5], bf16hi(a.z), s);
  s = fmaf(w[6], bf16lo(a.w), s);
  s = fmaf(w[7], bf16hi(a.w), s);
  s = fmaf(w[8], bf16lo(b.x), s);
  s = fmaf(w[9], bf16hi(b.x), s);
  s = fmaf(w[10], bf16lo(b.y), s);
  s = fmaf(w[11], bf16hi(b.y), s);
  s = fmaf(w[12], bf16lo(b.z), s);
  s = fmaf(w[13], bf16hi(b.z), s);
  s = fmaf(w[14], bf16lo(b.w), s);
  s = fmaf(w[15], bf16hi(b.w), s);
  return s;
}

__device__ __forceinline__ void unpack16(const uint4 v, float (&w)[16]) {
  i8x4_to_f32(v.x, w[0], w[1], w[2], w[3]);
  i8x4_to_f32(v.y, w[4], w[5], w[6], w[7]);
  i8x4_to_f32(v.z, w[8], w[9], w[10], w[11]);
  i8x4_to_f32(v.w, w[12], w[13], w[14], w[15]);
}

__global__ void __launch_bounds__(kSimtWarps * 32) i8_gemv_simt(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                 int M, int K, const int8_t* __restrict__ q,
                                                                 const float* __restrict__ scales,
                                                                 const float* __restrict__ bias, int64_t N, void* y,
                                                                 int64_t ldy, int epi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool swiglu = epi == MG_EPI_SWIGLU_BF16;
  const int64_t nout = swiglu ? N / 2 : N;
  const int64_t o = (int64_t)blockIdx.x * kSimtWarps + warp;
  if (o >= nout) return;
  const int64_t r0 = swiglu ? swiglu_gate_row(o) : o;
  const int64_t r1 = swiglu ? r0 + 64 : r0;
  const int8_t* w0 = q + r0 * K;
  const int8_t* w1 = q + r1 * K;
  for (int m0 = 0; m0 < M; m0 += kSimtMC) {
    float a0[kSimtMC], a1[kSimtMC];
#pragma unroll
    for (int i = 0; i < kSimtMC; ++i) a0[i] = a1[i] = 0.f;
    for (int k = lane * 16; k < K; k += 512) {
      float wf0[16], wf1[16];
      unpack16(ldg_stream(w0 + k), wf0);
      if (swiglu) unpack16(ldg_stream(w1 + k), wf1);
#pragma unroll
      for (int i = 0; i < kSimtMC; ++i) {
        if (m0 + i < M) {
          const __nv_bfloat16* xp = x + (int64_t)(m0 + i) * ldx + k;
          a0[i] += dot16(wf0, xp);
          if (swiglu) a1[i] += dot16(wf1, xp);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kSimtMC; ++i) {
      a0[i] = warp_sum(a0[i]);
      if (swiglu) a1[i] = warp_sum(a1[i]);
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kSimtMC; ++i) {
        const int m = m0 + i;
        if (m >= M) break;
        float v0 = a0[i] * scales[r0] + (bias ? bias[r0] : 0.f);
        if (swiglu) {
          const float v1 = a1[i] * scales[r1] + (bias ? bias[r1] : 0.f);
          static_cast<__nv_bfloat16*>(y)[(int64_t)m * ldy + o] = __float2bfloat16_rn(silu_f(v0) * v1);
        } else {
          store_out(epi, y, (int64_t)m * ldy + o, v0);
        }
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// tcgen05 kernel
// ------------------------------------------------------------------------------------------------
constexpr int kBN = 128;          // weight rows per tile (MMA M)
constexpr int kBK = 128;          // K per pipeline stage
constexpr int kTcThreads = 192;   // warps 0-3 convert + epilogue, warp 4 TMA, warp 5 MMA
constexpr uint32_t kWStageBytes = kBN * kBK;  // int8 tile

template <int MP>
struct TcCfg {
  static constexpr int kStages = MP <= 32 ? 4 : (MP <= 64 ? 3 : 2);
  static constexpr uint32_t kXStageBytes = MP * kBK * 2;  // bf16
  static constexpr uint32_t kStageBytes = kWStageBytes + kXStageBytes;
  static constexpr uint32_t kPipeBytes = kStages * kStageBytes;
  static constexpr uint32_t kRedBytes = MP * kBN * 4;
  static constexpr uint32_t kMainBytes = kPipeBytes > kRedBytes ? kPipeBytes : kRedBytes;
  static constexpr uint32_t kBarOffset = kMainBytes;
  static constexpr uint32_t kSmemBytes = kMainBytes + 256 + 1024;  // barriers + alignment slack
  static constexpr uint32_t kAccCol = 128;                          // A buffers use columns [0,128)
  static constexpr uint32_t kTmemCols = (128 + MP) <= 256 ? 256 : 512;
  // D=fp32 (bit 4), A=B=bf16 (bits 7, 10), K-major A and B, N = MP, M = 128.
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MP >> 3) << 17) |
                                     ((uint32_t)(kBN >> 4) << 24);
};

// Shared-memory descriptor of a K-major, 128B-swizzled bf16 tile (8-row x 128 B atoms, 1024 B apart).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;             // SWIZZLE_128B
  return d;
}

template <int MP>
__global__ void __launch_bounds__(kTcThreads, 1)
    i8_gemm_tc(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, int M, int K,
               int64_t N, const float* __restrict__ scales, const float* __restrict__ bias, void* y, int64_t ldy,
               int epi, int split) {
  using C = TcCfg<MP>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;
  uint64_t* aempty = afull + 2;
  uint64_t* accfull = aempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accfull + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = split > 1 ? cluster_ctarank() : 0;
  const int tile = blockIdx.x / split;
  const int mtile = blockIdx.y;
  const int kb_total = (K + kBK - 1) / kBK;
  const int kb_begin = (int)((int64_t)crank * kb_total / split);
  const int kb_end = (int)((int64_t)(crank + 1) * kb_total / split);
  const int nk = kb_end - kb_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], 4);
      mbar_init(&aempty[b], 1);
    }
    mbar_init(accfull, 1);
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 5) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  bool ok = true;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % S;
        if (i >= S) ok = mbar_wait(&empty[s], ((i / S) - 1) & 1, 1);
        if (!ok) break;
        uint8_t* sw = smem + s * C::kStageBytes;
        uint8_t* sx = sw + kWStageBytes;
        const int k0 = (kb_begin + i) * kBK;
        mbar_arrive_expect_tx(&full[s], C::kStageBytes);
        tma_load_2d(sw, &tmap_w, &full[s], k0, tile * kBN);
        tma_load_2d(sx, &tmap_x, &full[s], k0, mtile * MP);
        tma_load_2d(sx + MP * 128, &tmap_x, &full[s], k0 + 64, mtile * MP);
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % S, ab = i & 1;
        ok = mbar_wait(&full[s], (i / S) & 1, 2) && mbar_wait(&afull[ab], (i >> 1) & 1, 3);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sx = smem_u32(smem + s * C::kStageBytes + kWStageBytes);
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j) {
          const uint32_t a_t = tmem + (uint32_t)(ab * 64 + j * 8);
          const uint64_t bd = desc_sw128(sx + (uint32_t)((j >> 2) * MP * 128 + (j & 3) * 32));
          tc_mma_ts(tmem + C::kAccCol, a_t, bd, C::kIdesc, (i > 0 || j > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);
        tc_commit(&aempty[ab]);
      }
      tc_commit(accfull);
    }
  } else {
    // ---------------- converters: int8 smem row -> bf16 TMEM lane ----------------
    const int t = threadIdx.x;  // weight row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % S, ab = i & 1;
      ok = mbar_wait(&full[s], (i / S) & 1, 4);
      if (ok && i >= 2) ok = mbar_wait(&aempty[ab], ((i >> 1) - 1) & 1, 5);
      if (!ok) break;
      const uint8_t* row = smem + s * C::kStageBytes + t * 128;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t r[32];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const int c = h * 4 + c4;
          const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ (t & 7)) << 4));
          i8x4_to_bf16x4(v.x, r[c4 * 8 + 0], r[c4 * 8 + 1]);
          i8x4_to_bf16x4(v.y, r[c4 * 8 + 2], r[c4 * 8 + 3]);
          i8x4_to_bf16x4(v.z, r[c4 * 8 + 4], r[c4 * 8 + 5]);
          i8x4_to_bf16x4(v.w, r[c4 * 8 + 6], r[c4 * 8 + 7]);
        }
        tmem_st32(tmem + lane_base + (uint32_t)(ab * 64 + h * 32), r);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        mbar_arrive(&afull[ab]);
      }
    }
  }

  // ---------------- epilogue: TMEM -> shared (fp32, [MP][128]) ----------------
  float* red = reinterpret_cast<float*>(smem);
  if (warp < 4) {
    const int t = threadIdx.x;
    if (nk > 0 && mbar_wait(accfull, 0, 6)) {
      tc_fence_after();
      const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
#pragma unroll 1
      for (int c0 = 0; c0 < MP; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + C::kAccCol + (uint32_t)c0, r);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) red[(c0 + j) * kBN + t] = __uint_as_float(r[j]);
      }
    } else {
      for (int c = 0; c < MP; ++c) red[c * kBN + t] = 0.f;
    }
    tc_fence_before();
  }
  if (split > 1) cluster_sync_all(); else __syncthreads();

  // ---------------- split-K reduction + epilogue ----------------
  if (warp < 4) {
    const int t = threadIdx.x;
    const int m_base = mtile * MP;
    const int m_valid = min(MP, M - m_base);
    const bool swiglu = epi == MG_EPI_SWIGLU_BF16;
    const uint32_t red_addr = smem_u32(red);
    for (int ml = (int)crank; ml < m_valid; ml += split) {
      const int m = m_base + ml;
      if (!swiglu) {
        const int64_t n = (int64_t)tile * kBN + t;
        float v = 0.f;
        for (int j = 0; j < split; ++j) {
          const uint32_t a = red_addr + (uint32_t)((ml * kBN + t) * 4);
          v += split > 1 ? ld_dsmem_f32(mapa_shared(a, j)) : red[ml * kBN + t];
        }
        if (n < N) store_out(epi, y, (int64_t)m * ldy + n, v * scales[n] + (bias ? bias[n] : 0.f));
      } else if (t < 64) {
        const int64_t rg = (int64_t)tile * kBN + t, ru = rg + 64;
        float g = 0.f, u = 0.f;
        for (int j = 0; j < split; ++j) {
          const uint32_t ag = red_addr + (uint32_t)((ml * kBN + t) * 4);
          const uint32_t au = ag + 64 * 4;
          g += split > 1 ? ld_dsmem_f32(mapa_shared(ag, j)) : red[ml * kBN + t];
          u += split > 1 ? ld_dsmem_f32(mapa_shared(au, j)) : red[ml * kBN + t + 64];
        }
        if (ru < N) {
          const float gv = g * scales[rg] + (bias ? bias[rg] : 0.f);
          const float uv = u * scales[ru] + (bias ? bias[ru] : 0.f);
          static_cast<__nv_bfloat16*>(y)[(int64_t)m * ldy + (int64_t)tile * 64 + t] =
              __float2bfloat16_rn(silu_f(gv) * uv);
        }
      }
    }
  }
  if (split > 1) cluster_sync_all(); else __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled_t get_encode_fn() {
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

int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  PFN_encodeTiled_t enc = get_encode_fn();
  if (!enc) return MG_ERR_CUDA;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MG_OK : MG_ERR_INVALID_ARG;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int auto_split(int64_t tiles, int kblocks, int ctas_per_sm) {
  const int64_t slots = (int64_t)sm_count() * ctas_per_sm;
  int s = (int)(slots / (tiles > 0 ? tiles : 1));
  s = s < 1 ? 1 : s;
  s = s > 8 ? 8 : s;
  const int max_by_k = kblocks / 2 > 0 ? kblocks / 2 : 1;
  return s > max_by_k ? max_by_k : s;
}

template <int MP>
int launch_tc(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
              const float* bias, int64_t n, void* y, int64_t ldy, int epi, int split, cudaStream_t st) {
  using C = TcCfg<MP>;
  static bool attr_done = false;
  if (!attr_done) {
    MG_CUDA_TRY(cudaFuncSetAttribute(i8_gemm_tc<MP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    attr_done = true;
  }
  CUtensorMap mw, mx;
  int rc = make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, (uint64_t)k, (uint64_t)n, (uint64_t)k, kBK, kBN);
  if (rc) return rc;
  rc = make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)k, (uint64_t)m, (uint64_t)ldx * 2, 64, MP);
  if (rc) return rc;
  const int64_t tiles = (n + kBN - 1) / kBN;
  const int kblocks = (int)((k + kBK - 1) / kBK);
  const int64_t mtiles = (m + MP - 1) / MP;
  if (split <= 0) split = auto_split(tiles * mtiles, kblocks, MP <= 128 ? 2 : 1);
  if (split > kblocks) split = kblocks;
  if (split < 1) split = 1;
  if (split > 8 || tiles * split > 0x7fffffff || mtiles > 65535) return MG_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * split), (unsigned)mtiles, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MG_CUDA_TRY(cudaLaunchKernelEx(&cfg, i8_gemm_tc<MP>, mw, mx, (int)m, (int)k, n, scales, bias, y, ldy, epi, split));
  return MG_OK;
}

int check_linear_args(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
                      int64_t n, const void* y, int64_t ldy, int epi) {
  if (m < 0 || k <= 0 || n <= 0 || !x || !q || !scales || !y) return MG_ERR_INVALID_ARG;
  if (k % 16 || ldx < k || ldx % 8) return MG_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15) return MG_ERR_INVALID_ARG;
  if (epi < MG_EPI_STORE_BF16 || epi > MG_EPI_GELU_BF16) return MG_ERR_INVALID_ARG;
  if (epi == MG_EPI_SWIGLU_BF16 && (n % 128 || ldy < n / 2)) return MG_ERR_INVALID_ARG;
  if (epi != MG_EPI_SWIGLU_BF16 && ldy < n) return MG_ERR_INVALID_ARG;
  if (k > 0x7fffffff || m > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  return MG_OK;
}

}  // namespace

extern "C" int mg_i8_linear_simt(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                                 const float* scales, const float* bias, int64_t n, void* y, int64_t ldy, int epi,
                                 void* stream) {
  int rc = check_linear_args(x, m, k, ldx, q, scales, n, y, ldy, epi);
  if (rc) return rc;
  if (m == 0) return MG_OK;
  const int64_t nout = epi == MG_EPI_SWIGLU_BF16 ? n / 2 : n;
  const int64_t blocks = (nout + kSimtWarps - 1) / kSimtWarps;
  if (blocks > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  i8_gemv_simt<<<(unsigned)blocks, kSimtWarps * 32, 0, mg_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, (int)m, (int)k, q, scales, bias, n, y, ldy, epi);
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_i8_linear_tc(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                               const float* scales, const float* bias, int64_t n, void* y, int64_t ldy, int epi,
                               int split_k, void* stream) {
  int rc = check_linear_args(x, m, k, ldx, q, scales, n, y, ldy, epi);
  if (rc) return rc;
  if (m == 0) return MG_OK;
  if (split_k < 0 || split_k > 8) return MG_ERR_INVALID_ARG;
  cudaStream_t st = mg_stream(stream);
  if (m <= 16) return launch_tc<16>(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, split_k, st);
  if (m <= 32) return launch_tc<32>(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, split_k, st);
  if (m <= 64) return launch_tc<64>(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, split_k, st);
  if (m <= 128) return launch_tc<128>(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, split_k, st);
  return launch_tc<256>(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, split_k, st);
}

extern "C" int mg_i8_linear(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
                            const float* bias, int64_t n, void* y, int64_t ldy, int epi, void* stream) {
  return mg_i8_linear_tc(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, 0, stream);
}
