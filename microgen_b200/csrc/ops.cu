// Per-row kernels of the decode step: the INT8 quantizer, norms, embedding,
// RoPE + paged KV append, greedy argmax, and the graph-loop advance.
#include "common.cuh"

namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0) r = warp_sum(r);
  if (threadIdx.x == 0) red[0] = r;
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0) r = warp_max(r);
  if (threadIdx.x == 0) red[0] = r;
  __syncthreads();
  return red[0];
}

// One CTA per weight row. Restates quantized.py:30-39 bit-exactly:
// max|w| is exact in any order, the divisions are IEEE (__fdiv_rn), rintf rounds half to even.
__global__ void quantize_rows_kernel(const float* __restrict__ w, int64_t k, int8_t* __restrict__ q,
                                     float* __restrict__ scales) {
  // no early trigger: a following linear may prefetch the weights this kernel writes
 
  griddep_wait();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float* wr = w + row * k;
  float mx = 0.f;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) mx = fmaxf(mx, fabsf(wr[i]));
  mx = block_reduce_max(mx, red);
  const float s = fmaxf(__fdiv_rn(mx, 127.0f), 1e-8f);
  if (threadIdx.x == 0) scales[row] = s;
  int8_t* qr = q + row * k;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
    float v = rintf(__fdiv_rn(wr[i], s));
    v = fminf(fmaxf(v, -128.f), 127.f);
    qr[i] = static_cast<int8_t>(static_cast<int>(v));
  }
}

// Row norms, single pass: every thread loads its float4s (row and weight) up front, the row
// statistic is block-reduced, and the output is written from registers. n % 4 == 0, n <= 4*256*kMaxV.
constexpr int kNormMaxV = 8;

__device__ __forceinline__ void store_bf16x4(__nv_bfloat16* p, float a, float b, float c, float d) {
  uint2 v;
  v.x = pack_bf16x2(a, b);
  v.y = pack_bf16x2(c, d);
  *reinterpret_cast<uint2*>(p) = v;
}

__global__ void __launch_bounds__(kRowThreads) rmsnorm_kernel(const float* __restrict__ h,
                                                               const float* __restrict__ w, int n, float eps,
                                                               __nv_bfloat16* __restrict__ x) {
  griddep_launch();
  griddep_wait();
  __shared__ float red[32];
  const int nv = n >> 2;
  const float4* hr = reinterpret_cast<const float4*>(h + (int64_t)blockIdx.x * n);
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4 hv[kNormMaxV], wv[kNormMaxV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxV; ++i) {
    const int idx = threadIdx.x + i * kRowThreads;
    if (idx < nv) {
      hv[i] = hr[idx];
      wv[i] = wr[idx];
      ss += hv[i].x * hv[i].x + hv[i].y * hv[i].y + hv[i].z * hv[i].z + hv[i].w * hv[i].w;
    }
  }
  ss = block_reduce_sum(ss, red);
  const float inv = rsqrtf(ss / (float)n + eps);
  __nv_bfloat16* xr = x + (int64_t)blockIdx.x * n;
#pragma unroll
  for (int i = 0; i < kNormMaxV; ++i) {
    const int idx = threadIdx.x + i * kRowThreads;
    if (idx < nv)
      store_bf16x4(xr + 4 * idx, wv[i].x * (hv[i].x * inv), wv[i].y * (hv[i].y * inv), wv[i].z * (hv[i].z * inv),
                   wv[i].w * (hv[i].w * inv));
  }
}

__global__ void __launch_bounds__(kRowThreads) layernorm_kernel(const float* __restrict__ h,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ b, int n, float eps,
                                                                 __nv_bfloat16* __restrict__ x) {
  griddep_launch();
  griddep_wait();
  __shared__ float red[32];
  const int nv = n >> 2;
  const float4* hr = reinterpret_cast<const float4*>(h + (int64_t)blockIdx.x * n);
  float4 hv[kNormMaxV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxV; ++i) {
    const int idx = threadIdx.x + i * kRowThreads;
    if (idx < nv) {
      hv[i] = hr[idx];
      s += hv[i].x + hv[i].y + hv[i].z + hv[i].w;
    }
  }
  const float mean = block_reduce_sum(s, red) / (float)n;
  float v = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxV; ++i) {
    const int idx = threadIdx.x + i * kRowThreads;
    if (idx < nv) {
      const float a = hv[i].x - mean, c = hv[i].y - mean, d = hv[i].z - mean, e = hv[i].w - mean;
      v += a * a + c * c + d * d + e * e;
    }
  }
  const float inv = rsqrtf(block_reduce_sum(v, red) / (float)n + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
  const float4* br = reinterpret_cast<const float4*>(b);
  __nv_bfloat16* xr = x + (int64_t)blockIdx.x * n;
#pragma unroll
  for (int i = 0; i < kNormMaxV; ++i) {
    const int idx = threadIdx.x + i * kRowThreads;
    if (idx < nv) {
      const float4 wv = wr[idx], bv = br[idx];
      store_bf16x4(xr + 4 * idx, (hv[i].x - mean) * inv * wv.x + bv.x, (hv[i].y - mean) * inv * wv.y + bv.y,
                   (hv[i].z - mean) * inv * wv.z + bv.z, (hv[i].w - mean) * inv * wv.w + bv.w);
    }
  }
}

__global__ void embed_kernel(const int32_t* __restrict__ tokens, const int32_t* __restrict__ positions,
                             const float* __restrict__ wte, const float* __restrict__ wpe, int hidden, int64_t vocab,
                             int max_pos, float* __restrict__ h) {
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x;
  const int tok = tokens[i];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) mg_record_error(MG_ERR_DEVICE, 100);
    return;
  }
  int pos = 0;
  if (wpe) {
    pos = positions[i];
    if (pos < 0 || pos >= max_pos) {
      if (threadIdx.x == 0) mg_record_error(MG_ERR_DEVICE, 101);
      return;
    }
  }
  const float* e = wte + (int64_t)tok * hidden;
  float* hr = h + (int64_t)i * hidden;
  for (int j = threadIdx.x; j < hidden; j += blockDim.x) hr[j] = e[j] + (wpe ? wpe[(int64_t)pos * hidden + j] : 0.f);
}

// One CTA per (token, head); thread j owns the rotate-half pair (j, j + d/2). Heads [0,hq) are
// queries, [hq,hq+hkv) keys, [hq+hkv, hq+2hkv) values. RoPE (HF apply_rotary_pos_emb) on q and k;
// k and v land in the token's paged slot.
__global__ void rope_kv_append_kernel(const float* __restrict__ qkv, int64_t ld_qkv,
                                      const int32_t* __restrict__ positions, const float* __restrict__ cos_sin,
                                      int max_pos, const int32_t* __restrict__ slots, int hq, int hkv, int d,
                                      float* __restrict__ q_out, __nv_bfloat16* __restrict__ k_pool,
                                      __nv_bfloat16* __restrict__ v_pool, int64_t num_blocks) {
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x, hd = blockIdx.y, j = threadIdx.x;
  const int half = d >> 1;
  if (j >= half) return;
  const float* src = qkv + (int64_t)i * ld_qkv + (int64_t)hd * d;
  float a = src[j], b = src[j + half];
  if (hd < hq + hkv && cos_sin) {
    const int pos = positions[i];
    if (pos < 0 || pos >= max_pos) {
      if (j == 0) mg_record_error(MG_ERR_DEVICE, 200);
      return;
    }
    const float* cs = cos_sin + (int64_t)pos * d;
    const float c = cs[j], s = cs[half + j];
    const float ra = a * c - b * s;
    const float rb = b * c + a * s;
    a = ra;
    b = rb;
  }
  if (hd < hq) {
    float* dst = q_out + ((int64_t)i * hq + hd) * d;
    dst[j] = a;
    dst[j + half] = b;
    return;
  }
  const int slot = slots[i];
  const int64_t blk = slot >> 4;
  if (slot < 0 || blk >= num_blocks) {
    if (j == 0) mg_record_error(MG_ERR_DEVICE, 201);
    return;
  }
  const bool is_k = hd < hq + hkv;
  const int kh = is_k ? hd - hq : hd - hq - hkv;
  __nv_bfloat16* dst = (is_k ? k_pool : v_pool) + ((blk * hkv + kh) * 16 + (slot & 15)) * (int64_t)d;
  dst[j] = __float2bfloat16_rn(a);
  dst[j + half] = __float2bfloat16_rn(b);
}

// INT8 paged KV: the same rotation, then each K and V vector (one token, one kv head) is quantized as
// KVCacheState stores it with quantize_kv (kv_cache.py:30-35, 114-120): s = max(max|x| / 127, 1e-8),
// code = clamp(round_half_even(x / s), -128, 127) — int8 codes into the pools, s into the scale arrays
// (fp32 [num_blocks, hkv, 16]) at the same slot. Every thread of a CTA takes part in the vector's max.
__global__ void rope_kv_append_kv8_kernel(const float* __restrict__ qkv, int64_t ld_qkv,
                                          const int32_t* __restrict__ positions, const float* __restrict__ cos_sin,
                                          int max_pos, const int32_t* __restrict__ slots, int hq, int hkv, int d,
                                          float* __restrict__ q_out, int8_t* __restrict__ k_pool,
                                          int8_t* __restrict__ v_pool, float* __restrict__ k_scales,
                                          float* __restrict__ v_scales, int64_t num_blocks) {
  __shared__ float red[32];
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x, hd = blockIdx.y, j = threadIdx.x;
  const int half = d >> 1;
  const bool act = j < half;
  const float* src = qkv + (int64_t)i * ld_qkv + (int64_t)hd * d;
  float a = act ? src[j] : 0.f, b = act ? src[j + half] : 0.f;
  if (hd < hq + hkv && cos_sin) {
    const int pos = positions[i];
    if (pos < 0 || pos >= max_pos) {
      if (j == 0) mg_record_error(MG_ERR_DEVICE, 200);
      return;
    }
    if (act) {
      const float* cs = cos_sin + (int64_t)pos * d;
      const float c = cs[j], sn = cs[half + j];
      const float ra = a * c - b * sn;
      const float rb = b * c + a * sn;
      a = ra;
      b = rb;
    }
  }
  if (hd < hq) {
    if (act) {
      float* dst = q_out + ((int64_t)i * hq + hd) * d;
      dst[j] = a;
      dst[j + half] = b;
    }
    return;
  }
  const int slot = slots[i];
  const int64_t blk = slot >> 4;
  if (slot < 0 || blk >= num_blocks) {
    if (j == 0) mg_record_error(MG_ERR_DEVICE, 201);
    return;
  }
  float mx = fmaxf(fabsf(a), fabsf(b));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((j & 31) == 0) red[j >> 5] = mx;
  __syncthreads();
  mx = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  const float sc = fmaxf(__fdiv_rn(mx, 127.f), 1e-8f);
  const bool is_k = hd < hq + hkv;
  const int kh = is_k ? hd - hq : hd - hq - hkv;
  const int64_t row = (blk * hkv + kh) * 16 + (slot & 15);
  if (act) {
    int8_t* dst = (is_k ? k_pool : v_pool) + row * (int64_t)d;
    dst[j] = (int8_t)fminf(fmaxf(rintf(__fdiv_rn(a, sc)), -128.f), 127.f);
    dst[j + half] = (int8_t)fminf(fmaxf(rintf(__fdiv_rn(b, sc)), -128.f), 127.f);
  }
  if (j == 0) (is_k ? k_scales : v_scales)[row] = sc;
}

// torch.argmax semantics: the first index holding the maximum, NaN counting as larger than every
// number (a row with a NaN gives its first NaN). A row is split over a cluster of kArgSplit CTAs
// (contiguous chunks, float4 loads where the row is 16-byte aligned); CTA 0 of the cluster merges the
// chunk results through distributed shared memory, smaller index on ties.
constexpr int kArgSplit = 8;
constexpr int kArgThreads = 512;

__device__ __forceinline__ void argmax_take(float v, int32_t i, float& best, int32_t& bi) {
  if (mg_argmax_better(v, i, best, bi)) {
    best = v;
    bi = i;
  }
}

__device__ __forceinline__ void warp_argmax(float& best, int32_t& bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_take(ov, oi, best, bi);
  }
}

__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const float* __restrict__ logits, int64_t n, int64_t ld,
                                                             int32_t* __restrict__ out) {
  griddep_launch();
  griddep_wait();
  __shared__ float sv[kArgThreads / 32];
  __shared__ int32_t si[kArgThreads / 32];
  __shared__ float cta_best;
  __shared__ int32_t cta_idx;
  const int part = (int)blockIdx.x;  // rank in the cluster
  const float* r = logits + (int64_t)blockIdx.y * ld;
  const int64_t chunk = ((n + kArgSplit - 1) / kArgSplit + 3) / 4 * 4;
  const int64_t lo = (int64_t)part * chunk, hi = lo + chunk < n ? lo + chunk : n;
  float best = -INFINITY;
  int32_t bi = 0x7fffffff;
  int64_t i0 = lo;
  if ((reinterpret_cast<uintptr_t>(r) & 15) == 0 && hi > lo) {  // lo is a multiple of 4
    const int64_t nv = (hi - lo) >> 2;
    const float4* r4 = reinterpret_cast<const float4*>(r + lo);
    for (int64_t j = threadIdx.x; j < nv; j += kArgThreads) {
      const float4 v = r4[j];
      const int32_t k = (int32_t)(lo + 4 * j);
      argmax_take(v.x, k, best, bi);
      argmax_take(v.y, k + 1, best, bi);
      argmax_take(v.z, k + 2, best, bi);
      argmax_take(v.w, k + 3, best, bi);
    }
    i0 = lo + 4 * nv;
  }
  for (int64_t i = i0 + threadIdx.x; i < hi; i += kArgThreads) argmax_take(r[i], (int32_t)i, best, bi);
  warp_argmax(best, bi);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    best = l < kArgThreads / 32 ? sv[l] : -INFINITY;
    bi = l < kArgThreads / 32 ? si[l] : 0x7fffffff;
    warp_argmax(best, bi);
    if (l == 0) {
      cta_best = best;
      cta_idx = bi;
    }
  }
  cluster_sync_all();
  if (part == 0 && w == 0) {
    best = -INFINITY;
    bi = 0x7fffffff;
    if (l < kArgSplit) {
      best = ld_dsmem_f32(mapa_shared(smem_u32(&cta_best), (uint32_t)l));
      bi = __float_as_int(ld_dsmem_f32(mapa_shared(smem_u32(&cta_idx), (uint32_t)l)));
    }
    warp_argmax(best, bi);
    if (l == 0) out[blockIdx.y] = bi == 0x7fffffff ? 0 : bi;
  }
  cluster_sync_all();  // the other CTAs' results stay readable until CTA 0 has read them
}

__global__ void decode_advance_kernel(int32_t* tokens, const int32_t* next_tokens, int32_t* positions,
                                      int32_t* ctx_lens, int32_t* slots, const int32_t* tables, int max_blocks,
                                      int b) {
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= b) return;
  tokens[i] = next_tokens[i];
  const int pos = positions[i] + 1;
  positions[i] = pos;
  ctx_lens[i] = pos + 1;
  const int lb = pos >> 4;
  if (lb >= max_blocks) {
    mg_record_error(MG_ERR_DEVICE, 300);
    slots[i] = -1;
    return;
  }
  slots[i] = tables[(int64_t)i * max_blocks + lb] * 16 + (pos & 15);
}

}  // namespace

extern "C" int mg_quantize_rows_i8(const float* w, int64_t n, int64_t k, int8_t* q, float* scales, void* stream) {
  if (n < 0 || k < 0 || (n > 0 && (!w || !q || !scales)) || n > 0x7fffffff) return MG_ERR_INVALID_ARG;
  if (n == 0) return MG_OK;
  MG_CUDA_TRY(mg_launch(quantize_rows_kernel, dim3((unsigned)n), dim3(kRowThreads), 0, mg_stream(stream), 1, w, k, q, scales));
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_rmsnorm(const float* h, const float* w, int m, int n, float eps, void* x, void* stream) {
  if (m < 0 || n <= 0 || n % 4 || n > 4 * kRowThreads * kNormMaxV || !h || !w || !x) return MG_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15)
    return MG_ERR_INVALID_ARG;
  if (m == 0) return MG_OK;
  MG_CUDA_TRY(mg_launch(rmsnorm_kernel, dim3(m), dim3(kRowThreads), 0, mg_stream(stream), 1, h, w, n, eps,
                        static_cast<__nv_bfloat16*>(x)));
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_layernorm(const float* h, const float* w, const float* bias, int m, int n, float eps, void* x,
                            void* stream) {
  if (m < 0 || n <= 0 || n % 4 || n > 4 * kRowThreads * kNormMaxV || !h || !w || !bias || !x)
    return MG_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(bias) |
       reinterpret_cast<uintptr_t>(x)) & 15)
    return MG_ERR_INVALID_ARG;
  if (m == 0) return MG_OK;
  MG_CUDA_TRY(mg_launch(layernorm_kernel, dim3(m), dim3(kRowThreads), 0, mg_stream(stream), 1, h, w, bias, n, eps,
                        static_cast<__nv_bfloat16*>(x)));
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_embed(const int32_t* tokens, const int32_t* positions, const float* wte, const float* wpe, int b,
                        int hidden, int64_t vocab, int max_pos, float* h, void* stream) {
  if (b < 0 || hidden <= 0 || vocab <= 0 || !tokens || !wte || !h || (wpe && (!positions || max_pos <= 0)))
    return MG_ERR_INVALID_ARG;
  if (b == 0) return MG_OK;
  MG_CUDA_TRY(mg_launch(embed_kernel, dim3(b), dim3(kRowThreads), 0, mg_stream(stream), 1, tokens, positions, wte, wpe,
                        hidden, vocab, max_pos, h));
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_rope_kv_append(const float* qkv, int64_t ld_qkv, const int32_t* positions, const float* cos_sin,
                                 int max_pos, const int32_t* slot_mapping, int b, int hq, int hkv, int d,
                                 float* q_out, void* k_pool, void* v_pool, int64_t num_blocks, void* stream) {
  if (b < 0 || hq <= 0 || hkv <= 0 || hq % hkv || d <= 0 || (d & 1) || !qkv || !slot_mapping || !q_out || !k_pool ||
      !v_pool || num_blocks <= 0 || ld_qkv < (int64_t)(hq + 2 * hkv) * d || (cos_sin && (!positions || max_pos <= 0)))
    return MG_ERR_INVALID_ARG;
  if (b == 0) return MG_OK;
  if (d > 2 * 1024) return MG_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)b, (unsigned)(hq + 2 * hkv));
  MG_CUDA_TRY(mg_launch(rope_kv_append_kernel, grid, dim3((d / 2 + 31) / 32 * 32), 0, mg_stream(stream), 1, qkv,
                        ld_qkv, positions, cos_sin, max_pos, slot_mapping, hq, hkv, d, q_out,
                        static_cast<__nv_bfloat16*>(k_pool), static_cast<__nv_bfloat16*>(v_pool), num_blocks));
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_rope_kv_append_kv8(const float* qkv, int64_t ld_qkv, const int32_t* positions,
                                     const float* cos_sin, int max_pos, const int32_t* slot_mapping, int b, int hq,
                                     int hkv, int d, float* q_out, int8_t* k_pool, int8_t* v_pool, float* k_scales,
                                     float* v_scales, int64_t num_blocks, void* stream) {
  if (b < 0 || hq <= 0 || hkv <= 0 || hq % hkv || d <= 0 || (d & 1) || !qkv || !slot_mapping || !q_out || !k_pool ||
      !v_pool || !k_scales || !v_scales || num_blocks <= 0 || ld_qkv < (int64_t)(hq + 2 * hkv) * d ||
      (cos_sin && (!positions || max_pos <= 0)))
    return MG_ERR_INVALID_ARG;
  if (b == 0) return MG_OK;
  if (d > 2 * 1024) return MG_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)b, (unsigned)(hq + 2 * hkv));
  MG_CUDA_TRY(mg_launch(rope_kv_append_kv8_kernel, grid, dim3((d / 2 + 31) / 32 * 32), 0, mg_stream(stream), 1, qkv,
                        ld_qkv, positions, cos_sin, max_pos, slot_mapping, hq, hkv, d, q_out, k_pool, v_pool,
                        k_scales, v_scales, num_blocks));
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_argmax_rows(const float* logits, int m, int64_t n, int64_t ld, int32_t* out, void* stream) {
  if (m < 0 || n <= 0 || ld < n || !logits || !out || n > 0x7fffffff) return MG_ERR_INVALID_ARG;
  if (m == 0) return MG_OK;
  if (m > 65535) return MG_ERR_UNSUPPORTED;
  MG_CUDA_TRY(mg_launch(argmax_kernel, dim3(kArgSplit, m), dim3(kArgThreads), 0, mg_stream(stream), kArgSplit, logits,
                        n, ld, out));
  MG_LAUNCH_CHECK();
  return MG_OK;
}

extern "C" int mg_decode_advance(int32_t* tokens, const int32_t* next_tokens, int32_t* positions, int32_t* ctx_lens,
                                 int32_t* slots, const int32_t* block_tables, int max_blocks, int b, void* stream) {
  if (b < 0 || max_blocks <= 0 || !tokens || !next_tokens || !positions || !ctx_lens || !slots || !block_tables)
    return MG_ERR_INVALID_ARG;
  if (b == 0) return MG_OK;
  MG_CUDA_TRY(mg_launch(decode_advance_kernel, dim3((b + 127) / 128), dim3(128), 0, mg_stream(stream), 1, tokens,
                        next_tokens, positions, ctx_lens, slots, block_tables, max_blocks, b));
  MG_LAUNCH_CHECK();
  return MG_OK;
}
