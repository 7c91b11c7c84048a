// Paged-KV decode attention (one query token per sequence) over 16-token blocks.
//
// Pools are bf16 [num_blocks, hkv, 16, d]: one (block, kv head) tile is 16*d contiguous
// elements. The query heads of one GQA group (hq/hkv <= 16) form the 16 rows of an
// m16n8k16 tile, so QKᵀ and PV run on the tensor cores and the kernel stays bound by
// the KV bytes it streams.
//
// One launch covers two kinds of CTAs:
//   * shared CTAs — one per (kv head, chunk of up to kChunk shared-prefix blocks). The
//     chunk is loaded once into shared memory and every sequence's query group is run
//     against it (rows = batch x group), so a prefix shared by the whole batch is read
//     from HBM once per batch instead of once per sequence.
//   * private CTAs — one per (sequence, kv head, split) over the sequence's own blocks.
//     Four warps take interleaved blocks, each with its own double-buffered tiles and
//     online-softmax state, merged at the end.
// Each CTA leaves (m, l, unnormalised O) per query head in a workspace slot, and a
// combine kernel merges the slots (log-sum-exp). With no shared prefix and one split
// the private CTA writes the normalised output itself.
#include "common.cuh"

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 8;  // shared-prefix blocks per shared CTA

template <int D>
struct AttnCfg {
  static constexpr int kStride = D + 8;                 // padded smem row (bf16): conflict-free ldmatrix
  static constexpr int kTile = 16 * kStride;            // elements of one 16-token tile
  static constexpr int kPrivBytes = kWarps * 2 * 2 * kTile * 2;  // per warp: 2 stages x (K,V)
  static constexpr int kSharedBytes = kChunk * 2 * kTile * 2;
  static constexpr int kMergeBytes = kWarps * 16 * (D + 2) * 4;
  static constexpr int kSmem = (kPrivBytes > kSharedBytes ? kPrivBytes : kSharedBytes) > kMergeBytes
                                   ? (kPrivBytes > kSharedBytes ? kPrivBytes : kSharedBytes)
                                   : kMergeBytes;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Issue the async copies of one 16-token (K, V) tile of kv head h into smem rows of stride kStride.
// Rows >= valid are zero-filled (never read from global).
template <int D>
__device__ __forceinline__ void load_tile(uint32_t ks, uint32_t vs, const __nv_bfloat16* kp, const __nv_bfloat16* vp,
                                          int64_t blk, int hkv, int h, int valid, int lane, int nthreads) {
  constexpr int kChunksPerRow = D / 8;  // 16-byte chunks
  const int64_t base = ((blk * hkv + h) * 16) * (int64_t)D;
  for (int c = lane; c < 16 * kChunksPerRow; c += nthreads) {
    const int row = c / kChunksPerRow, col = (c % kChunksPerRow) * 8;
    const bool ok = row < valid;
    const uint32_t off = (uint32_t)(row * AttnCfg<D>::kStride + col) * 2;
    cp_async16(ks + off, kp + base + row * D + col, ok);
    cp_async16(vs + off, vp + base + row * D + col, ok);
  }
}

// Online-softmax update of one 16-row query tile with one 16-token KV tile.
template <int D>
__device__ __forceinline__ void attend_tile(const uint32_t (&qa)[D / 16][4], uint32_t ks, uint32_t vs, int valid,
                                            float (&o)[D / 8][4], float (&m)[2], float (&l)[2], int lane) {
  constexpr int kS = AttnCfg<D>::kStride;
  float s[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
  const int j8 = lane >> 3, r8 = lane & 7;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t b0, b1, b2, b3;
    const int tok = (j8 >> 1) * 8 + r8, d = kk * 16 + (j8 & 1) * 8;
    ldsm_x4(ks + (uint32_t)(tok * kS + d) * 2, b0, b1, b2, b3);
    mma_bf16(s[0], qa[kk], b0, b1);
    mma_bf16(s[1], qa[kk], b2, b3);
  }
  const int tq = (lane & 3) * 2;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (nt * 8 + tq + (c & 1) >= valid) s[nt][c] = -INFINITY;
  float alpha[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float mx = fmaxf(fmaxf(s[0][2 * r], s[0][2 * r + 1]), fmaxf(s[1][2 * r], s[1][2 * r + 1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m[r], mx);
    alpha[r] = exp2f(m[r] - mn);
    float sum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][2 * r] = exp2f(s[nt][2 * r] - mn);
      s[nt][2 * r + 1] = exp2f(s[nt][2 * r + 1] - mn);
      sum += s[nt][2 * r] + s[nt][2 * r + 1];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l[r] = l[r] * alpha[r] + sum;
    m[r] = mn;
  }
#pragma unroll
  for (int dn = 0; dn < D / 8; ++dn) {
    o[dn][0] *= alpha[0];
    o[dn][1] *= alpha[0];
    o[dn][2] *= alpha[1];
    o[dn][3] *= alpha[1];
  }
  uint32_t pa[4];
  pa[0] = pack_bf16x2(s[0][0], s[0][1]);
  pa[1] = pack_bf16x2(s[0][2], s[0][3]);
  pa[2] = pack_bf16x2(s[1][0], s[1][1]);
  pa[3] = pack_bf16x2(s[1][2], s[1][3]);
#pragma unroll
  for (int d2 = 0; d2 < D / 16; ++d2) {
    uint32_t b0, b1, b2, b3;
    const int tok = (j8 & 1) * 8 + r8, d = d2 * 16 + (j8 >> 1) * 8;
    ldsm_x4_t(vs + (uint32_t)(tok * kS + d) * 2, b0, b1, b2, b3);
    mma_bf16(o[2 * d2], pa, b0, b1);
    mma_bf16(o[2 * d2 + 1], pa, b2, b3);
  }
}

// A fragments of 16 query rows: row r of the tile is (seq_of(r), head_of(r)); rows with
// seq < 0 are padding (zero). q is fp32 [b, hq, d]; qscale folds softmax scale * log2(e).
template <int D>
__device__ __forceinline__ void load_q(uint32_t (&qa)[D / 16][4], const float* q, int hq, int row_seq0,
                                       int row_head0, int row_seq1, int row_head1, float qscale, int lane) {
  const int c = (lane & 3) * 2;
  const float* q0 = row_seq0 >= 0 ? q + ((int64_t)row_seq0 * hq + row_head0) * D : nullptr;
  const float* q1 = row_seq1 >= 0 ? q + ((int64_t)row_seq1 * hq + row_head1) * D : nullptr;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int d0 = kk * 16 + c;
    float2 a = q0 ? *reinterpret_cast<const float2*>(q0 + d0) : make_float2(0.f, 0.f);
    float2 b = q1 ? *reinterpret_cast<const float2*>(q1 + d0) : make_float2(0.f, 0.f);
    float2 e = q0 ? *reinterpret_cast<const float2*>(q0 + d0 + 8) : make_float2(0.f, 0.f);
    float2 f = q1 ? *reinterpret_cast<const float2*>(q1 + d0 + 8) : make_float2(0.f, 0.f);
    qa[kk][0] = pack_bf16x2(a.x * qscale, a.y * qscale);
    qa[kk][1] = pack_bf16x2(b.x * qscale, b.y * qscale);
    qa[kk][2] = pack_bf16x2(e.x * qscale, e.y * qscale);
    qa[kk][3] = pack_bf16x2(f.x * qscale, f.y * qscale);
  }
}

struct AttnParams {
  const float* q;
  const __nv_bfloat16* kp;
  const __nv_bfloat16* vp;
  int64_t num_blocks;
  const int32_t* tables;
  int max_blocks;
  const int32_t* ctx;
  int b, hq, hkv, group;
  int n_shared;   // shared-prefix blocks
  int n_shared_ctas_per_head;
  int nsplit, bps;  // private splits and blocks per split
  int nslots;       // workspace slots per (seq, head) = shared chunks + nsplit
  float qscale;
  __nv_bfloat16* out;
  float* ws_o;  // [b, hq, nslots, d]
  float* ws_ml; // [b, hq, nslots, 2]
  bool direct;  // private CTA writes the final output
};

template <int D>
__device__ void private_cta(const AttnParams& p, int pair, int sp, uint8_t* smem) {
  using C = AttnCfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = pair / p.hkv, h = pair % p.hkv;
  const int ctx = p.ctx[seq];
  const int nblk = (ctx + 15) >> 4;
  const int b0 = p.n_shared + sp * p.bps;
  const int b1 = min(nblk, b0 + p.bps);
  const int32_t* table = p.tables + (int64_t)seq * p.max_blocks;
  if (ctx < 1 || nblk > p.max_blocks) {
    if (threadIdx.x == 0) mg_record_error(MG_ERR_DEVICE, 400);
  }

  uint32_t qa[D / 16][4];
  const int g0 = lane >> 2, g1 = g0 + 8;
  load_q<D>(qa, p.q, p.hq, g0 < p.group ? seq : -1, h * p.group + g0, g1 < p.group ? seq : -1, h * p.group + g1,
            p.qscale, lane);
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  const uint32_t wbase = smem_u32(smem) + (uint32_t)(warp * 2 * 2 * C::kTile * 2);
  auto kst = [&](int st) { return wbase + (uint32_t)(st * 2 * C::kTile * 2); };
  auto vst = [&](int st) { return kst(st) + (uint32_t)(C::kTile * 2); };
  auto fetch = [&](int j, int st) {
    int64_t phys = table[j];
    const int valid = min(16, ctx - j * 16);
    if (phys < 0 || phys >= p.num_blocks) {
      mg_record_error(MG_ERR_DEVICE, 401);
      phys = 0;
    }
    load_tile<D>(kst(st), vst(st), p.kp, p.vp, phys, p.hkv, h, valid, lane, 32);
  };
  const bool tables_ok = ctx >= 1 && nblk <= p.max_blocks;
  int j = b0 + warp;
  if (tables_ok && j < b1) fetch(j, 0);
  cp_async_commit();
  int st = 0;
  for (; tables_ok && j < b1; j += kWarps) {
    const int jn = j + kWarps;
    if (jn < b1) fetch(jn, st ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    attend_tile<D>(qa, kst(st), vst(st), min(16, ctx - j * 16), o, m, l, lane);
    __syncwarp();
    st ^= 1;
  }
  cp_async_wait<0>();
  __syncthreads();

  // merge the four warps' states through shared memory: [warp][row][D + 2]
  float* mg = reinterpret_cast<float*>(smem);
  const int c = (lane & 3) * 2;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g0 + r * 8;
    float* dst = mg + (warp * 16 + row) * (D + 2);
#pragma unroll
    for (int dn = 0; dn < D / 8; ++dn) {
      dst[dn * 8 + c] = o[dn][2 * r];
      dst[dn * 8 + c + 1] = o[dn][2 * r + 1];
    }
    if ((lane & 3) == 0) {
      dst[D] = m[r];
      dst[D + 1] = l[r];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.group * D; idx += kThreads) {
    const int row = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mg[(w * 16 + row) * (D + 2) + D]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float* src = mg + (w * 16 + row) * (D + 2);
      const float wgt = M == -INFINITY ? 0.f : exp2f(src[D] - M);
      L += src[D + 1] * wgt;
      O += src[d] * wgt;
    }
    const int head = h * p.group + row;
    if (p.direct) {
      p.out[((int64_t)seq * p.hq + head) * D + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
    } else {
      const int slot = p.n_shared_ctas_per_head + sp;
      const int64_t base = ((int64_t)seq * p.hq + head) * p.nslots + slot;
      p.ws_o[base * D + d] = O;
      if (d == 0) {
        p.ws_ml[base * 2] = M;
        p.ws_ml[base * 2 + 1] = L;
      }
    }
  }
}

template <int D>
__device__ void shared_cta(const AttnParams& p, int h, int chunk, uint8_t* smem) {
  using C = AttnCfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk0 = chunk * kChunk;
  const int nb = min(kChunk, p.n_shared - blk0);
  const uint32_t base = smem_u32(smem);
  // shared blocks are the first n_shared entries of every table; read them from sequence 0's table
  for (int i = 0; i < nb; ++i) {
    int64_t phys = p.tables[blk0 + i];
    if (phys < 0 || phys >= p.num_blocks) {
      if (threadIdx.x == 0) mg_record_error(MG_ERR_DEVICE, 402);
      phys = 0;
    }
    const uint32_t ks = base + (uint32_t)(i * 2 * C::kTile * 2);
    load_tile<D>(ks, ks + C::kTile * 2, p.kp, p.vp, phys, p.hkv, h, 16, threadIdx.x, kThreads);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int rows = p.b * p.group;
  const int ntiles = (rows + 15) / 16;
  const int c = (lane & 3) * 2;
  for (int t = warp; t < ntiles; t += kWarps) {
    const int r0 = t * 16 + (lane >> 2), r1 = r0 + 8;
    const int s0 = r0 < rows ? r0 / p.group : -1, s1 = r1 < rows ? r1 / p.group : -1;
    uint32_t qa[D / 16][4];
    load_q<D>(qa, p.q, p.hq, s0, h * p.group + (r0 % p.group), s1, h * p.group + (r1 % p.group), p.qscale, lane);
    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    for (int i = 0; i < nb; ++i) {
      const uint32_t ks = base + (uint32_t)(i * 2 * C::kTile * 2);
      attend_tile<D>(qa, ks, ks + C::kTile * 2, 16, o, m, l, lane);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = r ? r1 : r0;
      if (row >= rows) continue;
      const int seq = row / p.group, head = h * p.group + row % p.group;
      const int64_t slot = ((int64_t)seq * p.hq + head) * p.nslots + chunk;
      float* dst = p.ws_o + slot * D;
#pragma unroll
      for (int dn = 0; dn < D / 8; ++dn) {
        dst[dn * 8 + c] = o[dn][2 * r];
        dst[dn * 8 + c + 1] = o[dn][2 * r + 1];
      }
      if ((lane & 3) == 0) {
        p.ws_ml[slot * 2] = m[r];
        p.ws_ml[slot * 2 + 1] = l[r];
      }
    }
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads) paged_attn_kernel(const AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  griddep_launch();
  griddep_wait();
  const int n_shared_ctas = p.n_shared_ctas_per_head * p.hkv;
  if ((int)blockIdx.x < n_shared_ctas) {
    shared_cta<D>(p, blockIdx.x / p.n_shared_ctas_per_head, blockIdx.x % p.n_shared_ctas_per_head, smem);
  } else {
    const int i = blockIdx.x - n_shared_ctas;
    private_cta<D>(p, i / p.nsplit, i % p.nsplit, smem);
  }
}

template <int D>
__global__ void combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_ml, int nslots,
                               __nv_bfloat16* __restrict__ out) {
  griddep_launch();
  griddep_wait();
  const int64_t sh = blockIdx.x;  // seq * hq + head
  const int d = threadIdx.x;
  const float* ml = ws_ml + sh * nslots * 2;
  float M = -INFINITY;
  for (int s = 0; s < nslots; ++s) M = fmaxf(M, ml[2 * s]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < nslots; ++s) {
    const float w = M == -INFINITY ? 0.f : exp2f(ml[2 * s] - M);
    L += ml[2 * s + 1] * w;
    O += ws_o[(sh * nslots + s) * D + d] * w;
  }
  out[sh * D + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
}

struct Plan {
  int n_shared_ctas_per_head, nsplit, bps, nslots;
  bool direct;
  size_t ws_bytes;
};

int sm_count_attn() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

Plan make_plan(int b, int hq, int hkv, int d, int max_blocks, int n_shared) {
  Plan pl{};
  pl.n_shared_ctas_per_head = (n_shared + kChunk - 1) / kChunk;
  const int priv_max = max_blocks - n_shared > 0 ? max_blocks - n_shared : 1;
  const int pairs = b * hkv;
  const int target = 3 * sm_count_attn() - pl.n_shared_ctas_per_head * hkv;
  int nsplit = target > pairs ? (target + pairs - 1) / pairs : 1;
  const int max_split = (priv_max + kWarps - 1) / kWarps;
  nsplit = nsplit > max_split ? max_split : nsplit;
  nsplit = nsplit < 1 ? 1 : nsplit;
  pl.bps = (priv_max + nsplit - 1) / nsplit;
  pl.nsplit = (priv_max + pl.bps - 1) / pl.bps;
  pl.nslots = pl.n_shared_ctas_per_head + pl.nsplit;
  pl.direct = pl.nslots == 1;
  pl.ws_bytes = pl.direct ? 0 : (size_t)b * hq * pl.nslots * (size_t)(d + 2) * sizeof(float);
  return pl;
}

template <int D>
int launch_attn(AttnParams& p, const Plan& pl, cudaStream_t st) {
  static bool attr_done = false;
  if (!attr_done) {
    MG_CUDA_TRY(cudaFuncSetAttribute(paged_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     AttnCfg<D>::kSmem));
    attr_done = true;
  }
  const int64_t ctas = (int64_t)pl.n_shared_ctas_per_head * p.hkv + (int64_t)p.b * p.hkv * pl.nsplit;
  if (ctas > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  MG_CUDA_TRY(mg_launch(paged_attn_kernel<D>, dim3((unsigned)ctas), dim3(kThreads), AttnCfg<D>::kSmem, st, 1, p));
  if (!pl.direct) {
    MG_CUDA_TRY(mg_launch(combine_kernel<D>, dim3((unsigned)(p.b * p.hq)), dim3(D), 0, st, 1, p.ws_o, p.ws_ml,
                          pl.nslots, p.out));
  }
  return MG_OK;
}

}  // namespace

extern "C" int mg_paged_attn_workspace_bytes(int b, int hq, int hkv, int d, int max_blocks, int n_shared_blocks,
                                             size_t* bytes) {
  if (!bytes || b < 0 || hq <= 0 || hkv <= 0 || hq % hkv || max_blocks <= 0 || n_shared_blocks < 0 ||
      n_shared_blocks > max_blocks)
    return MG_ERR_INVALID_ARG;
  if (d != 32 && d != 64 && d != 128) return MG_ERR_UNSUPPORTED;
  *bytes = make_plan(b, hq, hkv, d, max_blocks, n_shared_blocks).ws_bytes;
  return MG_OK;
}

extern "C" int mg_paged_decode_attn(const float* q, const void* k_pool, const void* v_pool, int64_t num_blocks,
                                    const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens, int b,
                                    int hq, int hkv, int d, int n_shared_blocks, float scale, void* out,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  if (b < 0 || hq <= 0 || hkv <= 0 || hq % hkv || hq / hkv > 16 || max_blocks <= 0 || num_blocks <= 0 ||
      n_shared_blocks < 0 || n_shared_blocks > max_blocks || !q || !k_pool || !v_pool || !block_tables ||
      !ctx_lens || !out)
    return MG_ERR_INVALID_ARG;
  if (d != 32 && d != 64 && d != 128) return MG_ERR_UNSUPPORTED;
  if (b == 0) return MG_OK;
  const Plan pl = make_plan(b, hq, hkv, d, max_blocks, n_shared_blocks);
  if (pl.ws_bytes > 0 && (!workspace || workspace_bytes < pl.ws_bytes)) return MG_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) | reinterpret_cast<uintptr_t>(q)) & 15)
    return MG_ERR_INVALID_ARG;
  AttnParams p{};
  p.q = q;
  p.kp = static_cast<const __nv_bfloat16*>(k_pool);
  p.vp = static_cast<const __nv_bfloat16*>(v_pool);
  p.num_blocks = num_blocks;
  p.tables = block_tables;
  p.max_blocks = max_blocks;
  p.ctx = ctx_lens;
  p.b = b;
  p.hq = hq;
  p.hkv = hkv;
  p.group = hq / hkv;
  p.n_shared = n_shared_blocks;
  p.n_shared_ctas_per_head = pl.n_shared_ctas_per_head;
  p.nsplit = pl.nsplit;
  p.bps = pl.bps;
  p.nslots = pl.nslots;
  p.qscale = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ws_o = static_cast<float*>(workspace);
  p.ws_ml = pl.ws_bytes ? static_cast<float*>(workspace) + (size_t)b * hq * pl.nslots * d : nullptr;
  p.direct = pl.direct;
  cudaStream_t st = mg_stream(stream);
  if (d == 32) return launch_attn<32>(p, pl, st);
  return d == 64 ? launch_attn<64>(p, pl, st) : launch_attn<128>(p, pl, st);
}

// ------------------------------------------------------------------------------------------------
// Allocation-free variant: the split scratch lives in a file-scope device array.
// ------------------------------------------------------------------------------------------------
#include <mutex>

namespace {

// Every GPU that loads this library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[MG_ATTN_NOALLOC_SCRATCH_BYTES];

constexpr int kNoAllocMaxDevices = 64;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device. In host code the array's name is only a
// host-side stand-in, so the address is looked up once per device (with that device current) and kept.
int noalloc_scratch_address(void** out) {
  int dev = 0;
  MG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return MG_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    MG_CUDA_TRY(cudaGetSymbolAddress(&p, g_attn_noalloc_scratch));
    if (!p) return MG_ERR_CUDA;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return MG_OK;
}

}  // namespace

extern "C" int mg_paged_decode_attn_noalloc(const float* q, const void* k_pool, const void* v_pool,
                                            int64_t num_blocks, const int32_t* block_tables, int max_blocks,
                                            const int32_t* ctx_lens, int b, int hq, int hkv, int d,
                                            int n_shared_blocks, float scale, void* out, void* stream) {
  size_t need = 0;
  int rc = mg_paged_attn_workspace_bytes(b, hq, hkv, d, max_blocks, n_shared_blocks, &need);
  if (rc) return rc;
  if (need > (size_t)MG_ATTN_NOALLOC_SCRATCH_BYTES) return MG_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  rc = noalloc_scratch_address(&scratch);
  if (rc) return rc;
  // Every split slot the combine step reads is written by this call's attention CTAs first, so the
  // previous call's contents never need clearing.
  return mg_paged_decode_attn(q, k_pool, v_pool, num_blocks, block_tables, max_blocks, ctx_lens, b, hq, hkv, d,
                              n_shared_blocks, scale, out, scratch, (size_t)MG_ATTN_NOALLOC_SCRATCH_BYTES, stream);
}
