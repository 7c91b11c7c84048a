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
//     warp 8      TMA-loads the int8 weight tile [128 rows x 128 B] (128B-swizzled) into
//                 the weight ring and the activation tile [MP x 128] bf16 (two 64-wide
//                 swizzled boxes) into the activation ring;
//     warps 0..7  (warp w: TMEM lane quarter w%4, K half w/4; thread <-> weight row) pull
//                 their bytes into registers (freeing the weight stage), convert them to
//                 bf16 (exact) and tcgen05.st them into a TMEM A buffer;
//     warp 9      issues 8 x tcgen05.mma kind::f16 (A from TMEM, B = activations
//                 from shared memory) accumulating fp32 into TMEM.
//   Split-K: the `split` CTAs of a thread-block cluster share one 128-row tile and
//   divide its K blocks; after the mainloop each CTA parks its fp32 accumulator in
//   shared memory and the cluster reduces it through distributed shared memory
//   (fixed order, deterministic), applying scale, bias and the epilogue — or, for a
//   row-parallel linear, pushing the tile into every rank's receive slot (comm.cu).
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace {

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float gelu_tanh_f(float v) {
  return 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
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
  griddep_launch();
  griddep_wait();
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
constexpr int kConvWarps = 8;     // warp w converts rows 32*(w%4).. (its TMEM lane quarter), K half w/4
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kTcThreads = 320;
constexpr uint32_t kWStageBytes = kBN * kBK;  // int8 tile
constexpr int kRedLoads = 16;                 // split-K partial loads in flight per thread

template <int MP>
struct TcCfg {
  // Weight ring (16 KB int8 stages, freed as soon as the converters hold the bytes in registers)
  // and activation ring (MP x 128 bf16 stages, freed by the MMA commit), sized to ~96 KB per CTA so
  // two CTAs share an SM for MP <= 128 (one CTA with ~192 KB for MP = 256).
  static constexpr int kWStages = MP <= 32 ? 5 : (MP <= 64 ? 4 : (MP <= 128 ? 2 : 4));
  static constexpr int kXStages = MP <= 16 ? 3 : 2;
  static constexpr int kABufs = MP <= 64 ? 3 : 2;                   // bf16 A tiles in TMEM (64 columns each)
  static constexpr uint32_t kXStageBytes = MP * kBK * 2;            // bf16
  static constexpr uint32_t kXOffset = kWStages * kWStageBytes;
  static constexpr uint32_t kPipeBytes = kXOffset + kXStages * kXStageBytes;
  static constexpr uint32_t kRedBytes = MP * kBN * 4;
  static constexpr uint32_t kMainBytes = kPipeBytes > kRedBytes ? kPipeBytes : kRedBytes;
  static constexpr uint32_t kBarOffset = kMainBytes;
  static constexpr uint32_t kSmemBytes = kBarOffset + 256 + 1024;  // barriers + alignment slack
  static constexpr uint32_t kAccCol = kABufs * 64;
  static constexpr uint32_t kTmemCols = (kAccCol + MP) <= 256 ? 256 : 512;
  // D=fp32 (bit 4), A=B=bf16 (bits 7, 10), K-major A and B, N = MP, M = 128.
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MP >> 3) << 17) |
                                     ((uint32_t)(kBN >> 4) << 24);
};

// Split-K reduction of one thread's columns ml0, ml0 + 2S, ... (< m_valid) at weight row r0: the
// S partials of each column come from the `red` buffers of the S CTAs of the cluster (fixed CTA
// order). Loads are issued in batches of about kRedLoads before any is consumed, so a batch costs
// one distributed-shared-memory latency.
template <int S, int MP, bool SWI, typename Emit>
__device__ __forceinline__ void reduce_cols(uint32_t red_addr, int r0, int ml0, int m_valid, Emit& emit) {
  constexpr int kCols = MP / (2 * S) > 0 ? MP / (2 * S) : 1;
  constexpr int kPer = S * (SWI ? 2 : 1);
  constexpr int kCB = kRedLoads / kPer > 0 ? (kRedLoads / kPer < kCols ? kRedLoads / kPer : kCols) : 1;
  uint32_t base[S];
#pragma unroll
  for (int j = 0; j < S; ++j) base[j] = S > 1 ? mapa_shared(red_addr, (uint32_t)j) : red_addr;
#pragma unroll 1
  for (int c0 = 0; c0 < kCols; c0 += kCB) {
    float p0[kCB][S], p1[kCB][SWI ? S : 1];
#pragma unroll
    for (int c = 0; c < kCB; ++c) {
      const int ml = ml0 + (c0 + c) * 2 * S;
      const bool ok = c0 + c < kCols && ml < m_valid;
#pragma unroll
      for (int j = 0; j < S; ++j) {
        const uint32_t a = base[j] + (uint32_t)((ml * kBN + r0) * 4);
        p0[c][j] = ok ? ld_dsmem_f32(a) : 0.f;
        if (SWI) p1[c][j] = ok ? ld_dsmem_f32(a + 64 * 4) : 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < kCB; ++c) {
      const int ml = ml0 + (c0 + c) * 2 * S;
      if (c0 + c < kCols && ml < m_valid) {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int j = 0; j < S; ++j) {
          a0 += p0[c][j];
          if (SWI) a1 += p1[c][j];
        }
        emit(ml, a0, a1);
      }
    }
  }
}

// Any other split (an explicit split_k of 3, 5, 6 or 7): one column at a time.
template <typename Emit>
__device__ __forceinline__ void reduce_cols_any(uint32_t red_addr, int r0, int ml0, int m_valid, int split,
                                                bool swiglu, Emit& emit) {
  for (int ml = ml0; ml < m_valid; ml += 2 * split) {
    const uint32_t off = (uint32_t)((ml * kBN + r0) * 4);
    float p0[8], p1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      p0[j] = 0.f;
      p1[j] = 0.f;
      if (j < split) {
        const uint32_t a = mapa_shared(red_addr, (uint32_t)j) + off;
        p0[j] = ld_dsmem_f32(a);
        if (swiglu) p1[j] = ld_dsmem_f32(a + 64 * 4);
      }
    }
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < split) {
        a0 += p0[j];
        a1 += p1[j];
      }
    }
    emit(ml, a0, a1);
  }
}

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
__global__ void __launch_bounds__(kTcThreads, 2)
    i8_gemm_tc(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, int M, int K,
               int64_t N, const float* __restrict__ scales, const float* __restrict__ bias, void* y, int64_t ldy,
               int epi, int split, int packed, const PeerOut po) {
  using C = TcCfg<MP>;
  constexpr int SW = C::kWStages;
  constexpr int SX = C::kXStages;
  constexpr int NA = C::kABufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* wempty = wfull + SW;
  uint64_t* xfull = wempty + SW;
  uint64_t* xempty = xfull + SX;
  uint64_t* afull = xempty + SX;
  uint64_t* aempty = afull + NA;
  uint64_t* accfull = aempty + NA;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accfull + 1);

  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = split > 1 ? cluster_ctarank() : 0;
  const int tile = blockIdx.x / split;
  const int mtile = blockIdx.y;
  const int kb_total = (K + kBK - 1) / kBK;
  const int kb_begin = (int)((int64_t)crank * kb_total / split);
  const int kb_end = (int)((int64_t)(crank + 1) * kb_total / split);
  const int nk = kb_end - kb_begin;
  // Weight tile (tile, kb): row-major codes -> box at (kb*128, tile*128); tile-packed codes (every
  // 128x128 tile stored as one contiguous 16 KB block) -> box at (0, (tile*kb_total + kb)*128).
  auto w_c0 = [&](int kb) { return packed ? 0 : kb * kBK; };
  auto w_c1 = [&](int kb) { return packed ? (tile * kb_total + kb) * kBN : tile * kBN; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kConvWarps);
    }
    for (int s = 0; s < SX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&afull[b], kConvWarps);
      mbar_init(&aempty[b], 1);
    }
    mbar_init(accfull, 1);
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  bool ok = true;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer: one thread feeding both rings ----------------
    if (lane == 0) {
      // Weight tiles do not depend on the previous kernel: the first weight stages are in flight
      // before the wait on the predecessor; activation tiles are only loaded after it.
      int iw = 0, ix = 0;
      for (; iw < nk && iw < SW; ++iw) {
        mbar_arrive_expect_tx(&wfull[iw], kWStageBytes);
        tma_load_2d(smem + iw * kWStageBytes, &tmap_w, &wfull[iw], w_c0(kb_begin + iw), w_c1(kb_begin + iw));
      }
      griddep_wait();
      uint32_t polls = 0;
      while ((iw < nk || ix < nk) && ok) {
        bool progressed = false;
        if (ix < nk && (ix < SX || mbar_test_wait(&xempty[ix % SX], ((ix / SX) - 1) & 1))) {
          const int s = ix % SX;
          uint8_t* sx = smem + C::kXOffset + s * C::kXStageBytes;
          const int k0 = (kb_begin + ix) * kBK;
          mbar_arrive_expect_tx(&xfull[s], C::kXStageBytes);
          tma_load_2d(sx, &tmap_x, &xfull[s], k0, mtile * MP);
          tma_load_2d(sx + MP * 128, &tmap_x, &xfull[s], k0 + 64, mtile * MP);
          ++ix;
          progressed = true;
        }
        if (iw < nk && mbar_test_wait(&wempty[iw % SW], ((iw / SW) - 1) & 1)) {
          const int s = iw % SW;
          mbar_arrive_expect_tx(&wfull[s], kWStageBytes);
          tma_load_2d(smem + s * kWStageBytes, &tmap_w, &wfull[s], w_c0(kb_begin + iw), w_c1(kb_begin + iw));
          ++iw;
          progressed = true;
        }
        if (!progressed) {
          if (++polls > MG_SPIN_LIMIT) {
            mg_record_error(MG_ERR_TIMEOUT, 1);
            ok = false;
          }
          __nanosleep(32);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % SX, ab = i % NA;
        ok = mbar_wait(&xfull[s], (i / SX) & 1, 2) && mbar_wait(&afull[ab], (i / NA) & 1, 3);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sx = smem_u32(smem + C::kXOffset + s * C::kXStageBytes);
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j) {
          const uint32_t a_t = tmem + (uint32_t)(ab * 64 + j * 8);
          const uint64_t bd = desc_sw128(sx + (uint32_t)((j >> 2) * MP * 128 + (j & 3) * 32));
          tc_mma_ts(tmem + C::kAccCol, a_t, bd, C::kIdesc, (i > 0 || j > 0) ? 1u : 0u);
        }
        tc_commit(&xempty[s]);
        tc_commit(&aempty[ab]);
      }
      tc_commit(accfull);
    }
  } else {
    // ---------------- converters: half an int8 smem row -> 32 bf16x2 TMEM columns ----------------
    const int row = (warp & 3) * 32 + lane;   // weight row within the tile == TMEM lane
    const int hh = warp >> 2;                 // K half: bytes [64*hh, 64*hh + 64)
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % SW, ab = i % NA;
      ok = mbar_wait(&wfull[s], (i / SW) & 1, 4);
      if (!ok) break;
      const uint8_t* src = smem + s * kWStageBytes + row * 128;
      uint4 v[4];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) v[c4] = *reinterpret_cast<const uint4*>(src + (((hh * 4 + c4) ^ (row & 7)) << 4));
      uint32_t r[32];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        i8x4_to_bf16x4(v[c4].x, r[c4 * 8 + 0], r[c4 * 8 + 1]);
        i8x4_to_bf16x4(v[c4].y, r[c4 * 8 + 2], r[c4 * 8 + 3]);
        i8x4_to_bf16x4(v[c4].z, r[c4 * 8 + 4], r[c4 * 8 + 5]);
        i8x4_to_bf16x4(v[c4].w, r[c4 * 8 + 6], r[c4 * 8 + 7]);
      }
      // the bytes have been consumed (converted): the stage can refill. Releasing it right after the shared
      // loads were issued could let the next TMA write land before a load returned.
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[s]);
      if (i >= NA) ok = mbar_wait(&aempty[ab], ((i / NA) - 1) & 1, 5);
      if (!ok) break;
      tmem_st32(tmem + lane_base + (uint32_t)(ab * 64 + hh * 32), r);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ab]);
    }
  }

  // ---------------- epilogue: TMEM -> shared (fp32, [MP][128]) ----------------
  griddep_wait();  // (returns at once: the producer already waited) every thread orders its y access
  float* red = reinterpret_cast<float*>(smem);
  constexpr int kColsPerWarp = MP >= 64 ? MP / 2 : MP;  // warps 4-7 take the upper half when MP >= 64
  if (warp < kConvWarps && (MP >= 64 || warp < 4)) {
    const int row = (warp & 3) * 32 + lane;
    const int c_begin = MP >= 64 ? (warp >> 2) * kColsPerWarp : 0;
    if (nk > 0 && mbar_wait(accfull, 0, 6)) {
      tc_fence_after();
      const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
#pragma unroll 1
      for (int c0 = c_begin; c0 < c_begin + kColsPerWarp; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + C::kAccCol + (uint32_t)c0, r);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < c_begin + kColsPerWarp) red[(c0 + j) * kBN + row] = __uint_as_float(r[j]);
      }
    } else {
      for (int c = c_begin; c < c_begin + kColsPerWarp; ++c) red[c * kBN + row] = 0.f;
    }
    tc_fence_before();
  }
  if (split > 1) cluster_sync_all(); else __syncthreads();
  if (warp == kMmaWarp) {  // the accumulator is out of TMEM
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }

  // ---------------- split-K reduction + epilogue ----------------
  // CTA `crank` owns token columns ml ≡ crank (mod split); within the CTA, converter thread t takes
  // weight row t % 128 and every second owned column (t / 128). For SwiGLU only rows < 64 are
  // active, each reducing its gate/up pair (t, t+64). A thread's (column, split) partials are read
  // through distributed shared memory in batches (reduce_cols); each column sums its partials in
  // fixed CTA order (deterministic). The residual add is a fire-and-forget reduction into y: exactly one thread
  // adds to each element, so the result does not depend on timing.
  if (warp < kConvWarps) {
    const int t = threadIdx.x;
    const int half = t >> 7;
    const int m_base = mtile * MP;
    const int m_valid = min(MP, M - m_base);
    const bool swiglu = epi == MG_EPI_SWIGLU_BF16;
    const uint32_t red_addr = smem_u32(red);
    const int r0 = swiglu ? (t & 63) : (t & 127);
    const int64_t n0 = (int64_t)tile * kBN + r0;
    const int64_t n1 = n0 + 64;  // SwiGLU up row
    const bool active = swiglu ? ((t & 127) < 64 && n1 < N) : (n0 < N);
    const float s0 = active ? scales[n0] : 0.f;
    const float b0 = (active && bias) ? bias[n0] : 0.f;
    const float s1 = (active && swiglu) ? scales[n1] : 0.f;
    const float b1 = (active && swiglu && bias) ? bias[n1] : 0.f;
    // Row-parallel push: the partial of all-reduce e goes to slot [e%2][rank] of every rank, each
    // word tagged with e. The previous push finished before this grid's dependency wait returned.
    const bool peer = epi == MG_EPI_PEER_F32;
    const uint32_t epoch = peer ? *reinterpret_cast<volatile uint32_t*>(po.count) + 1u : 0u;
    const uint64_t tag = (uint64_t)epoch << 32;
    const int ml0 = (int)crank + half * split;
    auto emit = [&](int ml, float a0, float a1) {
      const int m = m_base + ml;
      if (peer) {  // warp-uniform (N % 128 == 0): lane pairs (n, n+1) share one word
        const float v = a0 * s0;
        const float v1 = __shfl_down_sync(0xffffffffu, v, 1);
        if ((n0 & 1) == 0) {
          const uint64_t word = tag | pack_bf16x2(v, v1);
          const int64_t off = ((int64_t)(epoch & 1u) * po.world + po.rank) * po.slot + ((int64_t)m * N + n0) / 2;
          for (int r = 0; r < po.world; ++r) st_volatile_u64(po.recv[r] + off, word);
        }
      } else if (epi == MG_EPI_ADD_F32) {
        red_add_f32(static_cast<float*>(y) + (int64_t)m * ldy + n0, a0 * s0 + b0);
      } else if (!swiglu) {
        store_out(epi, y, (int64_t)m * ldy + n0, a0 * s0 + b0);
      } else {
        const float gv = a0 * s0 + b0, uv = a1 * s1 + b1;
        static_cast<__nv_bfloat16*>(y)[(int64_t)m * ldy + (int64_t)tile * 64 + r0] =
            __float2bfloat16_rn(silu_f(gv) * uv);
      }
    };
    if (active) {
#define MG_RED(S)                                                                                      \
  (swiglu ? reduce_cols<S, MP, true>(red_addr, r0, ml0, m_valid, emit)                                  \
          : reduce_cols<S, MP, false>(red_addr, r0, ml0, m_valid, emit))
      switch (split) {
        case 1: MG_RED(1); break;
        case 2: MG_RED(2); break;
        case 4: MG_RED(4); break;
        case 8: MG_RED(8); break;
        default: reduce_cols_any(red_addr, r0, ml0, m_valid, split, swiglu, emit); break;
      }
#undef MG_RED
    }
  }
  if (split > 1) {
    cluster_sync_all();  // peers may still be reading this CTA's partials
  } else if (epi == MG_EPI_PEER_F32) {
    __syncthreads();     // every thread has read the count
  }
  // The last CTA to finish advances this rank's all-reduce count, which the reduce kernel (the next
  // grid) reads as the epoch to wait for. Every CTA read the count before counting itself.
  if (epi == MG_EPI_PEER_F32 && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(po.done, 1u) == gridDim.x * gridDim.y - 1u) {
      *reinterpret_cast<volatile uint32_t*>(po.done) = 0u;
      *reinterpret_cast<volatile uint32_t*>(po.count) += 1u;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Stream-K form of the tcgen05 kernel (tile-packed codes, m <= 128).
//
// The work of one launch is the list of units (weight tile t, K block kb) in the order u = t*KB + kb,
// which is also the order of the tile-packed codes in memory. The grid is one resident wave of CTAs
// (SMs x CTAs per SM, at most one CTA per two units) and CTA c streams the contiguous units
// [c*U/G, (c+1)*U/G): every CTA gets the same number of weight bytes, so no SM idles on a short tile
// count or a partial second wave, and no thread-block cluster or distributed shared memory is needed.
//
// A CTA's range is a sequence of segments (its units of one tile). The MMA warp accumulates a segment
// in TMEM; at the segment's end the converter warps drain the accumulator into shared memory (the MMA
// warp then starts the next segment) and
//   * a segment that is the whole tile runs the epilogue directly;
//   * a segment that does not start at the tile's first K block (only a CTA's first segment can be one)
//     stores its fp32 partial in the workspace slot of this CTA and raises the CTA's flag;
//   * a segment that starts the tile but ends before its last K block belongs to the tile's finisher:
//     it waits for the flags of the following CTAs whose first segment lies in the tile, adds their
//     partials in CTA order (the sum does not depend on timing) and runs the epilogue.
// The finisher reaches such a tile at the end of its own range, the contributors at the start of theirs,
// so the wait is normally already satisfied. All CTAs of the grid are resident together, so the waits
// cannot deadlock; every wait is still bounded (MG_ERR_TIMEOUT). The finisher clears the flags it
// consumed, so the workspace is left as it was found (zero flags): it must be zero-filled before its
// first use and may be shared by any stream-ordered sequence of launches.
// ------------------------------------------------------------------------------------------------
template <int MP>
struct SkCfg {
  static constexpr int kCtasPerSm = MP <= 32 ? 2 : 1;
  static constexpr int kWStages = MP <= 16 ? 5 : (MP <= 32 ? 4 : (MP <= 64 ? 8 : 6));
  static constexpr int kXStages = MP <= 64 ? 3 : 2;
  static constexpr int kABufs = MP <= 32 ? 3 : (MP <= 64 ? 6 : 4);
  static constexpr uint32_t kXStageBytes = MP * kBK * 2;
  static constexpr uint32_t kXOffset = kWStages * kWStageBytes;
  static constexpr uint32_t kRedOffset = kXOffset + kXStages * kXStageBytes;
  static constexpr uint32_t kRedBytes = MP * kBN * 4;
  static constexpr uint32_t kBarOffset = kRedOffset + kRedBytes;
  static constexpr uint32_t kSmemBytes = kBarOffset + 512 + 1024;  // barriers + alignment slack
  static constexpr uint32_t kAccCol = kABufs * 64;
  static constexpr uint32_t kTmemCols = kCtasPerSm == 2 ? 256 : 512;
  static constexpr uint32_t kIdesc = TcCfg<MP>::kIdesc;
  static_assert(kAccCol + (MP < 32 ? 32 : MP) <= kTmemCols, "TMEM columns");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
  static_assert(kCtasPerSm == 1 || 2 * (kSmemBytes + 1024) <= 228 * 1024, "two CTAs per SM");
  static_assert((2 * kWStages + 2 * kXStages + 2 * kABufs + 2) * 8 + 4 <= 512, "barrier region");
};

__device__ __forceinline__ void conv_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Converter-warp barrier that also returns whether every converter thread passed `ok`.
__device__ __forceinline__ bool conv_bar_and(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int MP>
__global__ void __launch_bounds__(kTcThreads, SkCfg<MP>::kCtasPerSm)
    i8_gemm_sk(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, int M, int K,
               int64_t N, const float* __restrict__ scales, const float* __restrict__ bias, void* y, int64_t ldy,
               int epi, const PeerOut po, float* __restrict__ part, uint32_t* __restrict__ flags) {
  using C = SkCfg<MP>;
  constexpr int SW = C::kWStages;
  constexpr int SX = C::kXStages;
  constexpr int NA = C::kABufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* wempty = wfull + SW;
  uint64_t* xfull = wempty + SW;
  uint64_t* xempty = xfull + SX;
  uint64_t* afull = xempty + SX;
  uint64_t* aempty = afull + NA;
  uint64_t* accfull = aempty + NA;
  uint64_t* accempty = accfull + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accempty + 1);
  float* red = reinterpret_cast<float*>(smem + C::kRedOffset);
  __shared__ int s_ok;  // the finisher's flag wait succeeded

  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (K + kBK - 1) / kBK;
  const int64_t U = ((N + kBN - 1) / kBN) * KB;
  const int G = gridDim.x, cta = blockIdx.x;
  auto ubeg = [&](int c) { return (int64_t)c * U / G; };
  const int64_t u0 = ubeg(cta), u1 = ubeg(cta + 1);
  const int nk = (int)(u1 - u0);
  // segment boundaries: the segment containing stage i ends at stage seg_last(i)
  auto seg_last = [&](int i) {
    const int64_t tile_end = ((u0 + i) / KB + 1) * KB;
    return (int)(min(u1, tile_end) - u0) - 1;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kConvWarps);
    }
    for (int s = 0; s < SX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&afull[b], kConvWarps);
      mbar_init(&aempty[b], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(accempty, 1);
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // Weight stages (the tile-packed unit u is the 16 KB block at row u*128) do not depend on the
      // previous kernel and are issued before the dependency wait; activation stages after it.
      bool ok = true;
      int iw = 0, ix = 0;
      for (; iw < nk && iw < SW; ++iw) {
        mbar_arrive_expect_tx(&wfull[iw], kWStageBytes);
        tma_load_2d(smem + iw * kWStageBytes, &tmap_w, &wfull[iw], 0, (int)((u0 + iw) * kBN));
      }
      griddep_wait();
      uint32_t polls = 0;
      while ((iw < nk || ix < nk) && ok) {
        bool progressed = false;
        if (ix < nk && (ix < SX || mbar_test_wait(&xempty[ix % SX], ((ix / SX) - 1) & 1))) {
          const int s = ix % SX;
          uint8_t* sx = smem + C::kXOffset + s * C::kXStageBytes;
          const int k0 = (int)((u0 + ix) % KB) * kBK;
          mbar_arrive_expect_tx(&xfull[s], C::kXStageBytes);
          tma_load_2d(sx, &tmap_x, &xfull[s], k0, 0);
          tma_load_2d(sx + MP * 128, &tmap_x, &xfull[s], k0 + 64, 0);
          ++ix;
          progressed = true;
        }
        if (iw < nk && mbar_test_wait(&wempty[iw % SW], ((iw / SW) - 1) & 1)) {
          const int s = iw % SW;
          mbar_arrive_expect_tx(&wfull[s], kWStageBytes);
          tma_load_2d(smem + s * kWStageBytes, &tmap_w, &wfull[s], 0, (int)((u0 + iw) * kBN));
          ++iw;
          progressed = true;
        }
        if (!progressed) {
          if (++polls > MG_SPIN_LIMIT) {
            mg_record_error(MG_ERR_TIMEOUT, 11);
            ok = false;
          }
          __nanosleep(32);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      bool ok = true;
      int seg = 0;
      for (int i = 0; i < nk && ok;) {
        const int first = i, last = seg_last(i);
        if (seg > 0) {  // the previous segment's accumulator has been drained
          ok = mbar_wait(accempty, (seg - 1) & 1, 12);
          if (!ok) break;
          tc_fence_after();
        }
        for (; i <= last && ok; ++i) {
          const int s = i % SX, ab = i % NA;
          ok = mbar_wait(&xfull[s], (i / SX) & 1, 13) && mbar_wait(&afull[ab], (i / NA) & 1, 14);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sx = smem_u32(smem + C::kXOffset + s * C::kXStageBytes);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            const uint32_t a_t = tmem + (uint32_t)(ab * 64 + j * 8);
            const uint64_t bd = desc_sw128(sx + (uint32_t)((j >> 2) * MP * 128 + (j & 3) * 32));
            tc_mma_ts(tmem + C::kAccCol, a_t, bd, C::kIdesc, (i > first || j > 0) ? 1u : 0u);
          }
          tc_commit(&xempty[s]);
          tc_commit(&aempty[ab]);
        }
        if (ok) tc_commit(accfull);
        ++seg;
      }
    }
  } else {
    // ---------------- converters, then each segment's epilogue ----------------
    const int row = (warp & 3) * 32 + lane;
    const int hh = warp >> 2;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const bool swiglu = epi == MG_EPI_SWIGLU_BF16;
    const bool peer = epi == MG_EPI_PEER_F32;
    const int t = threadIdx.x;
    const int half = t >> 7;
    const int r0 = swiglu ? (t & 63) : (t & 127);
    const int m_valid = min(MP, M);
    bool ok = true, waited = false;
    uint32_t epoch = 0;
    int seg = 0;
    for (int i = 0; i < nk;) {
      const int last = seg_last(i);
      const int64_t useg = u0 + i;
      const int64_t tile = useg / KB;
      for (; i <= last; ++i) {
        const int s = i % SW, ab = i % NA;
        if (ok) ok = mbar_wait(&wfull[s], (i / SW) & 1, 15);
        // the TMEM buffer is claimed before the stage is read, so no converted registers stay live across a wait
        if (ok && i >= NA) ok = mbar_wait(&aempty[ab], ((i / NA) - 1) & 1, 16);
        uint4 v[4];
        uint32_t r[32];
        if (ok) {
          const uint8_t* src = smem + s * kWStageBytes + row * 128;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            v[c4] = *reinterpret_cast<const uint4*>(src + (((hh * 4 + c4) ^ (row & 7)) << 4));
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            i8x4_to_bf16x4(v[c4].x, r[c4 * 8 + 0], r[c4 * 8 + 1]);
            i8x4_to_bf16x4(v[c4].y, r[c4 * 8 + 2], r[c4 * 8 + 3]);
            i8x4_to_bf16x4(v[c4].z, r[c4 * 8 + 4], r[c4 * 8 + 5]);
            i8x4_to_bf16x4(v[c4].w, r[c4 * 8 + 6], r[c4 * 8 + 7]);
          }
        }
        // released only after the bytes were consumed (converted), see the cluster kernel's converters
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&wempty[s]);
        if (ok) {
          tmem_st32(tmem + lane_base + (uint32_t)(ab * 64 + hh * 32), r);
          tc_wait_st();
          tc_fence_before();
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&afull[ab]);
      }
      // ---- segment epilogue: drain the accumulator into `red` [col][row] ----
      if (ok) ok = mbar_wait(accfull, seg & 1, 17);
      constexpr int kColsPerWarp = MP >= 64 ? MP / 2 : MP;
      if (ok && (MP >= 64 || warp < 4)) {
        tc_fence_after();
        const int c_begin = MP >= 64 ? (warp >> 2) * kColsPerWarp : 0;
#pragma unroll 1
        for (int c0 = c_begin; c0 < c_begin + kColsPerWarp; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + C::kAccCol + (uint32_t)c0, r);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < c_begin + kColsPerWarp) red[(c0 + j) * kBN + row] = __uint_as_float(r[j]);
        }
        tc_fence_before();
      }
      if (!conv_bar_and(ok)) {
        ok = false;
        break;  // uniform across the converter warps
      }
      if (t == 0) mbar_arrive(accempty);  // the MMA warp may overwrite the accumulator
      if (!waited) {
        griddep_wait();  // (already satisfied) orders this thread's reads/writes of y after the predecessor
        waited = true;
        if (peer) epoch = *reinterpret_cast<volatile uint32_t*>(po.count) + 1u;
      }
      const bool starts = useg % KB == 0;
      const bool ends = (u0 + last + 1) % KB == 0;
      if (!starts) {
        // contributor: this CTA's partial of the tile into its workspace slot, then its flag. The
        // barrier orders every thread's stores before thread 0's release (cumulative at GPU scope).
        float4* dst = reinterpret_cast<float4*>(part + (int64_t)cta * MP * kBN);
        const float4* srcv = reinterpret_cast<const float4*>(red);
        for (int idx = t; idx < MP * kBN / 4; idx += 256) __stcg(dst + idx, srcv[idx]);
        conv_bar_sync();
        if (t == 0) st_release_u32(flags + cta, 1u);
      } else {
        if (!ends) {
          // finisher: the following CTAs whose first segment lies in this tile each left a partial.
          // Thread j polls contributor j's flag (all at once), then every thread adds, for its own
          // elements, the partials in CTA order (fixed order: bit-reproducible).
          const int64_t tile_end = (tile + 1) * KB;
          int nc = 0;
          while (cta + 1 + nc < G && ubeg(cta + 1 + nc) < tile_end) ++nc;
          if (t == 0) s_ok = 1;
          conv_bar_sync();
          if (t < nc) {
            uint32_t* f = flags + cta + 1 + t;
            uint64_t t0 = 0;
            for (uint32_t spin = 0; ld_acquire_u32(f) == 0u; ++spin) {
              if ((spin & 31) == 31) {
                const uint64_t now = global_ns();
                if (t0 == 0) {
                  t0 = now;
                } else if (now - t0 > 1000000000ull) {
                  mg_record_error(MG_ERR_TIMEOUT, 18);
                  s_ok = 0;
                  break;
                }
                __nanosleep(64);
              }
            }
            *f = 0u;  // consumed (the next launch's writers run after this grid completed)
          }
          conv_bar_sync();
          if (!s_ok) ok = false;
          constexpr int kBatch = 8;  // partial loads in flight per thread
          float4* acc4 = reinterpret_cast<float4*>(red);
          for (int idx = t; idx < MP * kBN / 4; idx += 256) {
            float4 acc = acc4[idx];
            for (int j0 = 0; j0 < nc; j0 += kBatch) {
              float4 v[kBatch];
#pragma unroll
              for (int j = 0; j < kBatch; ++j)
                if (j0 + j < nc) v[j] = __ldcg(reinterpret_cast<const float4*>(part + (int64_t)(cta + 1 + j0 + j) * MP * kBN) + idx);
#pragma unroll
              for (int j = 0; j < kBatch; ++j) {
                if (j0 + j < nc) {
                  acc.x += v[j].x;
                  acc.y += v[j].y;
                  acc.z += v[j].z;
                  acc.w += v[j].w;
                }
              }
            }
            acc4[idx] = acc;
          }
          conv_bar_sync();
        }
        // epilogue of the whole tile from `red`: thread t takes weight row r0 and every second token
        // column from `half` (SwiGLU: rows < 64 pair gate row r0 with up row r0 + 64)
        const int64_t n0 = tile * kBN + r0;
        const int64_t n1 = n0 + 64;
        const bool active = swiglu ? ((t & 127) < 64 && n1 < N) : (n0 < N);
        if (active) {
          const float s0 = scales[n0];
          const float b0 = bias ? bias[n0] : 0.f;
          const float s1 = swiglu ? scales[n1] : 0.f;
          const float b1 = (swiglu && bias) ? bias[n1] : 0.f;
          const uint64_t tag = (uint64_t)epoch << 32;
          for (int ml = half; ml < m_valid; ml += 2) {
            const float a0 = red[ml * kBN + r0];
            if (peer) {  // warp-uniform (N % 128 == 0): lane pairs (n, n+1) share one word
              const float v = a0 * s0;
              const float v1 = __shfl_down_sync(0xffffffffu, v, 1);
              if ((n0 & 1) == 0) {
                const uint64_t word = tag | pack_bf16x2(v, v1);
                const int64_t off = ((int64_t)(epoch & 1u) * po.world + po.rank) * po.slot + ((int64_t)ml * N + n0) / 2;
                for (int r = 0; r < po.world; ++r) st_volatile_u64(po.recv[r] + off, word);
              }
            } else if (epi == MG_EPI_ADD_F32) {
              red_add_f32(static_cast<float*>(y) + (int64_t)ml * ldy + n0, a0 * s0 + b0);
            } else if (!swiglu) {
              store_out(epi, y, (int64_t)ml * ldy + n0, a0 * s0 + b0);
            } else {
              const float gv = a0 * s0 + b0, uv = red[ml * kBN + r0 + 64] * s1 + b1;
              static_cast<__nv_bfloat16*>(y)[(int64_t)ml * ldy + tile * 64 + r0] =
                  __float2bfloat16_rn(silu_f(gv) * uv);
            }
          }
        }
      }
      conv_bar_sync();  // `red` is free for the next segment
      ++seg;
    }
    if (!waited) griddep_wait();
  }
  __syncthreads();
  if (warp == kMmaWarp) {  // every accumulator has been drained
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  // The last CTA to finish advances this rank's all-reduce count (read by the reduce kernel).
  if (epi == MG_EPI_PEER_F32 && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(po.done, 1u) == gridDim.x - 1u) {
      *reinterpret_cast<volatile uint32_t*>(po.done) = 0u;
      *reinterpret_cast<volatile uint32_t*>(po.count) += 1u;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------------
int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  return mg_make_map_2d(map, dt, base, inner, outer, row_bytes, box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
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

// Split-K factor: the largest power of two (cluster of 1, 2, 4 or 8 CTAs) with tiles x split within
// one wave of resident CTAs and at least two K blocks per CTA. Power-of-two clusters pack the GPCs
// without leftover SMs; a cluster that does not fit waits for a second wave.
int auto_split(int64_t tiles, int kblocks, int ctas_per_sm) {
  const int64_t slots = (int64_t)sm_count() * ctas_per_sm;
  int s = 1;
  while (s < 8 && tiles * (s * 2) <= slots && kblocks >= 4 * s) s *= 2;
  return s;
}

template <int MP>
int launch_tc(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
              const float* bias, int64_t n, void* y, int64_t ldy, int epi, int split, cudaStream_t st,
              bool packed, const PeerOut* po) {
  using C = TcCfg<MP>;
  static bool attr_done[64] = {};
  static std::mutex attr_mu;
  MG_CUDA_TRY(mg_once_per_device(attr_done, attr_mu, [] {
    return cudaFuncSetAttribute(i8_gemm_tc<MP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  }));
  CUtensorMap mw, mx;
  const uint64_t packed_rows = (uint64_t)((n + kBN - 1) / kBN) * ((k + kBK - 1) / kBK) * kBN;
  int rc = packed ? make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, kBK, packed_rows, kBK, kBK, kBN)
                  : make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, (uint64_t)k, (uint64_t)n, (uint64_t)k, kBK, kBN);
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
  MG_CUDA_TRY(mg_launch(i8_gemm_tc<MP>, dim3((unsigned)(tiles * split), (unsigned)mtiles, 1), dim3(kTcThreads),
                        C::kSmemBytes, st, (unsigned)split, mw, mx, (int)m, (int)k, n, scales, bias, y, ldy, epi,
                        split, packed ? 1 : 0, po ? *po : PeerOut{}));
  return MG_OK;
}

int dispatch_tc(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
                const float* bias, int64_t n, void* y, int64_t ldy, int epi, int split_k, cudaStream_t st,
                bool packed, const PeerOut* po = nullptr) {
#define MG_TC(MPV) launch_tc<MPV>(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, split_k, st, packed, po)
  if (m <= 16) return MG_TC(16);
  if (m <= 32) return MG_TC(32);
  if (m <= 64) return MG_TC(64);
  if (m <= 128) return MG_TC(128);
  return MG_TC(256);
#undef MG_TC
}

// ---- stream-K dispatch (tile-packed codes, m <= 128) ----
int sk_mp(int64_t m) { return m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : (m <= 128 ? 128 : 0))); }
int sk_ctas_per_sm(int mp) { return mp <= 32 ? 2 : 1; }
constexpr int64_t kSkMinUnits = 2;  // K blocks per CTA at least (fewer, bigger CTAs for small linears)
size_t sk_flag_bytes(int64_t grid) { return (size_t)((grid * 4 + 255) / 256 * 256); }
size_t sk_ws_bytes(int mp, int64_t grid) { return sk_flag_bytes(grid) + (size_t)grid * mp * kBN * 4; }

template <int MP>
int launch_sk(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed, const float* scales,
              const float* bias, int64_t n, void* y, int64_t ldy, int epi, void* ws, size_t ws_bytes,
              cudaStream_t st, const PeerOut* po) {
  using C = SkCfg<MP>;
  static bool attr_done[64] = {};
  static std::mutex attr_mu;
  MG_CUDA_TRY(mg_once_per_device(attr_done, attr_mu, [] {
    return cudaFuncSetAttribute(i8_gemm_sk<MP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  }));
  const int64_t tiles = (n + kBN - 1) / kBN, kblocks = (k + kBK - 1) / kBK, units = tiles * kblocks;
  int64_t grid = (int64_t)sm_count() * C::kCtasPerSm;
  grid = std::min(grid, std::max<int64_t>(1, units / kSkMinUnits));
  if (units * kBN > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  if (!ws || ws_bytes < sk_ws_bytes(MP, grid) || (reinterpret_cast<uintptr_t>(ws) & 255)) return MG_ERR_INVALID_ARG;
  CUtensorMap mw, mx;
  int rc = make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, kBK, (uint64_t)(units * kBN), kBK, kBK, kBN);
  if (rc) return rc;
  rc = make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)k, (uint64_t)m, (uint64_t)ldx * 2, 64, MP);
  if (rc) return rc;
  uint32_t* flags = static_cast<uint32_t*>(ws);
  float* part = reinterpret_cast<float*>(static_cast<char*>(ws) + sk_flag_bytes(grid));
  MG_CUDA_TRY(mg_launch(i8_gemm_sk<MP>, dim3((unsigned)grid), dim3(kTcThreads), C::kSmemBytes, st, 1, mw, mx, (int)m,
                        (int)k, n, scales, bias, y, ldy, epi, po ? *po : PeerOut{}, part, flags));
  return MG_OK;
}

int dispatch_sk(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed, const float* scales,
                const float* bias, int64_t n, void* y, int64_t ldy, int epi, void* ws, size_t ws_bytes,
                cudaStream_t st, const PeerOut* po = nullptr) {
  switch (sk_mp(m)) {
    case 16: return launch_sk<16>(x, m, k, ldx, packed, scales, bias, n, y, ldy, epi, ws, ws_bytes, st, po);
    case 32: return launch_sk<32>(x, m, k, ldx, packed, scales, bias, n, y, ldy, epi, ws, ws_bytes, st, po);
    case 64: return launch_sk<64>(x, m, k, ldx, packed, scales, bias, n, y, ldy, epi, ws, ws_bytes, st, po);
    case 128: return launch_sk<128>(x, m, k, ldx, packed, scales, bias, n, y, ldy, epi, ws, ws_bytes, st, po);
    default: return dispatch_tc(x, m, k, ldx, packed, scales, bias, n, y, ldy, epi, 0, st, true, po);
  }
}

// [tiles][kblocks][128 rows][128 B]: packed[((t*KB + kb)*128 + r)*128 + c] = q[(t*128 + r)*k + kb*128 + c],
// zero where the row or column is past the matrix. One thread per 16 bytes.
__global__ void pack_tiles_kernel(const int8_t* __restrict__ q, int64_t n, int64_t k, int8_t* __restrict__ out,
                                  int64_t total16) {
  griddep_wait();  // no early trigger: the linears that follow prefetch these codes before waiting
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total16) return;
  const int64_t kb_total = (k + kBK - 1) / kBK;
  const int64_t c16 = i & 7;          // 16-byte chunk within the 128-byte tile row
  const int64_t r = (i >> 3) & 127;   // tile row
  const int64_t blk = i >> 10;        // t * KB + kb
  const int64_t t = blk / kb_total, kb = blk % kb_total;
  const int64_t row = t * kBN + r, col = kb * kBK + c16 * 16;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (row < n && col < k) v = *reinterpret_cast<const uint4*>(q + row * k + col);  // k % 16 == 0
  reinterpret_cast<uint4*>(out)[i] = v;
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
  MG_CUDA_TRY(mg_launch(i8_gemv_simt, dim3((unsigned)blocks), dim3(kSimtWarps * 32), 0, mg_stream(stream), 1,
                        static_cast<const __nv_bfloat16*>(x), ldx, (int)m, (int)k, q, scales, bias, n, y, ldy, epi));
  return MG_OK;
}

extern "C" int mg_i8_linear_tc(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                               const float* scales, const float* bias, int64_t n, void* y, int64_t ldy, int epi,
                               int split_k, void* stream) {
  int rc = check_linear_args(x, m, k, ldx, q, scales, n, y, ldy, epi);
  if (rc) return rc;
  if (m == 0) return MG_OK;
  if (split_k < 0 || split_k > 8) return MG_ERR_INVALID_ARG;
  return dispatch_tc(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, split_k, mg_stream(stream), false);
}

extern "C" int64_t mg_i8_packed_bytes(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0) return 0;
  return ((n + kBN - 1) / kBN) * kBN * ((k + kBK - 1) / kBK) * kBK;
}

extern "C" int mg_i8_pack_weights(const int8_t* q, int64_t n, int64_t k, int8_t* packed, void* stream) {
  if (!q || !packed || n <= 0 || k <= 0 || k % 16) return MG_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(packed)) & 15) return MG_ERR_INVALID_ARG;
  const int64_t total16 = mg_i8_packed_bytes(n, k) / 16;
  const int64_t blocks = (total16 + 255) / 256;
  if (blocks > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  MG_CUDA_TRY(mg_launch(pack_tiles_kernel, dim3((unsigned)blocks), dim3(256), 0, mg_stream(stream), 1, q, n, k,
                        packed, total16));
  return MG_OK;
}

extern "C" int mg_i8_linear_packed(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed,
                                   const float* scales, const float* bias, int64_t n, void* y, int64_t ldy, int epi,
                                   int split_k, void* stream) {
  int rc = check_linear_args(x, m, k, ldx, packed, scales, n, y, ldy, epi);
  if (rc) return rc;
  if (m == 0) return MG_OK;
  if (split_k < 0 || split_k > 8) return MG_ERR_INVALID_ARG;
  return dispatch_tc(x, m, k, ldx, packed, scales, bias, n, y, ldy, epi, split_k, mg_stream(stream), true);
}

extern "C" int mg_i8_linear(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
                            const float* bias, int64_t n, void* y, int64_t ldy, int epi, void* stream) {
  return mg_i8_linear_tc(x, m, k, ldx, q, scales, bias, n, y, ldy, epi, 0, stream);
}

extern "C" int mg_i8_linear_packed_rowpar(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed,
                                          const float* scales, int64_t n, void* comm, int split_k, void* stream) {
  PeerOut po;
  int rc = mg_comm_peer_out(comm, &po);
  if (rc) return rc;
  if (m < 0 || k <= 0 || n <= 0 || !x || !packed || !scales || k % 16 || n % 128 || ldx < k || ldx % 8 ||
      split_k < 0 || split_k > 8 || m * n > 2 * po.slot ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(packed)) & 15))
    return MG_ERR_INVALID_ARG;
  if (k > 0x7fffffff || m > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  if (m == 0) return MG_OK;
  return dispatch_tc(x, m, k, ldx, packed, scales, nullptr, n, nullptr, n, MG_EPI_PEER_F32, split_k,
                     mg_stream(stream), true, &po);
}

// ---- stream-K entry points ----------------------------------------------------------------------
extern "C" int64_t mg_i8_linear_sk_workspace_bytes(int64_t m) {
  const int mp = sk_mp(m);
  if (m <= 0 || !mp) return 0;
  return (int64_t)sk_ws_bytes(mp, (int64_t)sm_count() * sk_ctas_per_sm(mp));
}

extern "C" int mg_i8_linear_packed_sk(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed,
                                      const float* scales, const float* bias, int64_t n, void* y, int64_t ldy,
                                      int epi, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_linear_args(x, m, k, ldx, packed, scales, n, y, ldy, epi);
  if (rc) return rc;
  if (m == 0) return MG_OK;
  return dispatch_sk(x, m, k, ldx, packed, scales, bias, n, y, ldy, epi, workspace, workspace_bytes,
                     mg_stream(stream));
}

extern "C" int mg_i8_linear_packed_rowpar_sk(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed,
                                             const float* scales, int64_t n, void* comm, void* workspace,
                                             size_t workspace_bytes, void* stream) {
  PeerOut po;
  int rc = mg_comm_peer_out(comm, &po);
  if (rc) return rc;
  if (m < 0 || k <= 0 || n <= 0 || !x || !packed || !scales || k % 16 || n % 128 || ldx < k || ldx % 8 ||
      m * n > 2 * po.slot || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(packed)) & 15))
    return MG_ERR_INVALID_ARG;
  if (k > 0x7fffffff || m > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  if (m == 0) return MG_OK;
  return dispatch_sk(x, m, k, ldx, packed, scales, nullptr, n, nullptr, n, MG_EPI_PEER_F32, workspace,
                     workspace_bytes, mg_stream(stream), &po);
}
