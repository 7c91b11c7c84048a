// Paged-KV decode attention (one query token per sequence) over 16-token blocks.
//
// Pools are bf16 [num_blocks, hkv, 16, d]: one (block, kv head) tile is 16*d contiguous
// elements, i.e. 16 rows of a 2-D tensor [num_blocks*hkv*16, d] that TMA reads. The query
// heads of one GQA group (hq/hkv <= 16) form the 16 rows of an m16n8k16 tile, so QKᵀ and PV
// run on the tensor cores and the kernel stays bound by the KV bytes it streams.
//
// A CTA is one producer warp (TMA loads of (K, V) tiles into a ring of kStages shared-memory
// stages, 128-byte swizzled so the ldmatrix reads are conflict-free) and kCons consumer warps.
// One launch covers two kinds of CTAs:
//   * shared CTAs — one per (kv head, chunk of up to kChunk shared-prefix blocks, group of
//     kCons query row tiles). The chunk is loaded once and every sequence's query group is run
//     against it (rows = batch x group), so a prefix shared by the whole batch is read from HBM
//     once per batch instead of once per sequence.
//   * private CTAs — one per (sequence, kv head, split) over the sequence's own blocks. Tile i
//     of the split goes to stage i % kStages and consumer warp i % kCons (each warp owns
//     kStages/kCons stages, so that many of its tiles are in flight); each warp keeps its own
//     online-softmax state, merged at the end.
// Each CTA leaves (m, l, unnormalised O) per query head in a workspace slot, and a combine
// kernel merges the slots (log-sum-exp). With no shared prefix and one split the private CTA
// writes the normalised output itself.
//
// INT8 KV (Q8): pools are int8 [num_blocks, hkv, 16, d] with one fp32 scale per (block, kv head,
// token) vector for K and for V. A stage holds the int8 K and V tiles (TMA, swizzled) and their 16 + 16
// scales (bulk copies). Private CTAs of the transposed form feed the codes from the stage straight into f16
// MMA fragments (exact integer conversion in registers; K and V fragment orders chosen so ldmatrix can
// deliver them); the other forms convert the codes exactly to bf16 first (a warp into its own tile buffer,
// the shared CTA's warps together into a double buffer). Scales apply outside the MMAs: each score is
// multiplied by its key's scale, and each probability by its value's scale before the PV product (the
// softmax sum uses the unscaled probabilities).
#include <cuda_fp16.h>

#include "common.cuh"

namespace {

constexpr int kCons = 4;                 // consumer warps
constexpr int kProd = kCons;             // producer warp index
constexpr int kThreads = (kCons + 1) * 32;
constexpr int kStages = 8;               // KV ring stages (a multiple of kCons)
constexpr int kChunk = 8;                // shared-prefix blocks per shared CTA (<= kStages)
static_assert(kStages % kCons == 0 && kChunk <= kStages, "ring layout");

template <int D, bool Q8 = false>
struct AttnCfg {
  static constexpr int kBf16Tile = 16 * D * 2;                // bf16 K (or V) of one block and kv head
  static constexpr int kTileBytes = Q8 ? 16 * D : kBf16Tile;  // as stored in the pool
  static constexpr int kStageBytes = 2 * kTileBytes + (Q8 ? 128 : 0);
  // Q8 ring: kStages K tiles, then kStages V tiles (TMA-swizzled so ldmatrix reads them without bank
  // conflicts), then kStages x 128 bytes of scales (16 K scales, 16 V scales per stage)
  static constexpr int kVRing = kStages * kTileBytes;
  static constexpr int kSRing = 2 * kStages * kTileBytes;
  static constexpr int kRingBytes = Q8 ? kSRing + kStages * 128 : kStages * kStageBytes;
  static constexpr int kMergeBytes = kCons * 16 * (D + 2) * 4;
  static constexpr int kMain = kRingBytes > kMergeBytes ? kRingBytes : kMergeBytes;
  // Q8: converted bf16 tiles + their 32 scales, one buffer per consumer warp (the shared CTA uses two)
  static constexpr int kBufBytes = 2 * kBf16Tile + 128;
  static constexpr int kBufOffset = (kMain + 127) / 128 * 128;
  static constexpr int kBufTotal = Q8 ? kCons * kBufBytes : 0;
  static constexpr int kBarOffset = (kBufOffset + kBufTotal + 7) / 8 * 8;
  static constexpr int kSmem = kBarOffset + (2 * kStages + 1) * 8 + 1024;  // + 1 KB alignment slack
  static constexpr int kBoxCols = D >= 64 ? 64 : D;       // one bf16 TMA box row = 128 B (64 B for d = 32)
};

// Byte offset of (row, col) in a tile. d >= 64: halves of 64 columns, each 16 rows x 128 B with the
// 16-byte chunks XOR-swizzled by row % 8 (TMA SWIZZLE_128B); d = 32: plain 64-byte rows.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  if constexpr (D >= 64) {
    const int half = col >> 6, c = col & 63;
    return (uint32_t)(half * 2048 + row * 128 + ((((c >> 3) ^ (row & 7))) << 4) + (c & 7) * 2);
  } else {
    return (uint32_t)(row * D * 2 + col * 2);
  }
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
__device__ __forceinline__ void mma_f16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Four int8 codes -> four exact f16 values: the biased byte b + 128 becomes the low mantissa bits of
// 1024 (0x64 high byte), and 1152 is subtracted.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  const uint32_t a = __byte_perm(x, 0x64646464u, 0x4140), b = __byte_perm(x, 0x64646464u, 0x4342);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(0x64806480u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(0x64806480u));
}
// The four codes of a 16-bit-pair register (bytes: token a dim c, token a dim c+1, token b dim c, token b
// dim c+1) -> f16 pairs (dim c: tokens a, b) and (dim c+1: tokens a, b), exactly.
__device__ __forceinline__ void i8pairs_to_f16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  const uint32_t a = __byte_perm(x, 0x64646464u, 0x4240), b = __byte_perm(x, 0x64646464u, 0x4341);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(0x64806480u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(0x64806480u));
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMA loads of the K and V tiles of (block phys, kv head h) into one ring stage; with Q8 the int8
// tiles (one box of 16 rows x d bytes each) and the tiles' K and V scales (64 bytes each). ring: the
// CTA's ring base; s: the stage.
template <int D, bool Q8 = false>
__device__ __forceinline__ void load_stage(uint8_t* ring, int s, const CUtensorMap* tk, const CUtensorMap* tv,
                                           uint64_t* bar, int row, const float* k_scales = nullptr,
                                           const float* v_scales = nullptr) {
  using C = AttnCfg<D, Q8>;
  constexpr int T = C::kTileBytes;
  mbar_arrive_expect_tx(bar, C::kStageBytes);
  if constexpr (Q8) {
    tma_load_2d(ring + s * T, tk, bar, 0, row);
    tma_load_2d(ring + C::kVRing + s * T, tv, bar, 0, row);
    bulk_load_smem(ring + C::kSRing + s * 128, k_scales + row, 64, bar);
    bulk_load_smem(ring + C::kSRing + s * 128 + 64, v_scales + row, 64, bar);
  } else {
    uint8_t* st = ring + s * C::kStageBytes;
#pragma unroll
    for (int c = 0; c < D; c += C::kBoxCols) {
      tma_load_2d(st + c * 32, tk, bar, c, row);  // 16 rows x 128 B = 2 KB per 64 columns
      tma_load_2d(st + T + c * 32, tv, bar, c, row);
    }
  }
}

// Q8: byte offset of (row, byte) in a stage's int8 K tile, as TMA wrote it: 16 rows of d bytes with the
// 16-byte chunks XOR-swizzled (128/64/32-byte swizzle for d = 128/64/32: offset bits 4.. ^= bits 7..).
template <int D>
__device__ __forceinline__ uint32_t k8_off(int row, int byte) {
  constexpr uint32_t kMask = D == 128 ? 7u : (D == 64 ? 3u : 1u);
  const uint32_t o = (uint32_t)(row * D + byte);
  return o ^ (((o >> 7) & kMask) << 4);
}

// Q8: a stage's int8 tiles -> exact bf16 integers in the swizzled tile layout of the bf16 path at dst (K
// when with_k, then V at dst + one bf16 tile), and the stage's scales after them (V scales of tokens >=
// valid become 0, so a zero probability never meets a stale scale). Threads t, t + n, ... take part.
template <int D>
__device__ __forceinline__ void convert_stage(const uint8_t* ring, int s, uint8_t* dst, int valid, int t, int n,
                                              bool with_k) {
  using C = AttnCfg<D, true>;
  constexpr int kChunks = 16 * D / 16;  // 16-byte chunks per int8 tile
  const uint32_t dk = smem_u32(dst);
  const uint8_t* kt = ring + s * C::kTileBytes;
  const uint8_t* vt = ring + C::kVRing + s * C::kTileBytes;
  for (int c = with_k ? t : kChunks + t; c < 2 * kChunks; c += n) {
    const int kv = c >= kChunks, cc = c - kv * kChunks;
    const int row = cc / (D / 16), col = (cc % (D / 16)) * 16;
    const uint4 w = *reinterpret_cast<const uint4*>((kv ? vt : kt) + k8_off<D>(row, col));
    uint32_t r[8];
    i8x4_to_bf16x4(w.x, r[0], r[1]);
    i8x4_to_bf16x4(w.y, r[2], r[3]);
    i8x4_to_bf16x4(w.z, r[4], r[5]);
    i8x4_to_bf16x4(w.w, r[6], r[7]);
    const uint32_t base = dk + kv * C::kBf16Tile;
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(base + swz<D>(row, col)), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(base + swz<D>(row, col + 8)), "r"(r[4]), "r"(r[5]),
                 "r"(r[6]), "r"(r[7])
                 : "memory");
  }
  for (int j = t; j < 32; j += n) {
    const float v = reinterpret_cast<const float*>(ring + C::kSRing + s * 128)[j];
    reinterpret_cast<float*>(dst + 2 * C::kBf16Tile)[j] = (j >= 16 && j - 16 >= valid) ? 0.f : v;
  }
}

// Zero V rows [valid, 16) of a stage (a partial last block: those pool slots hold no token, and
// P = 0 there must not meet a NaN). The stage then goes back to the async proxy.
template <int D>
__device__ __forceinline__ void zero_v_tail(uint32_t vs, int valid, int lane) {
  constexpr int kChunksPerRow = D / 8;
  for (int c = valid * kChunksPerRow + lane; c < 16 * kChunksPerRow; c += 32) {
    const int row = c / kChunksPerRow, col = (c % kChunksPerRow) * 8;
    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vs + swz<D>(row, col)), "r"(0u) : "memory");
  }
  __syncwarp();
}

// Online-softmax update of one 16-row query tile with one 16-token KV tile.
template <int D>
__device__ __forceinline__ void attend_tile(const uint32_t (&qa)[D / 16][4], uint32_t ks, uint32_t vs, int valid,
                                            float (&o)[D / 8][4], float (&m)[2], float (&l)[2], int lane,
                                            const float* sc = nullptr) {
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
    ldsm_x4(ks + swz<D>(tok, d), b0, b1, b2, b3);
    mma_bf16(s[0], qa[kk], b0, b1);
    mma_bf16(s[1], qa[kk], b2, b3);
  }
  const int tq = (lane & 3) * 2;
  if (sc) {  // Q8: key scales (score column nt * 8 + tq + (c & 1) is that key)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[nt][c] *= sc[nt * 8 + tq + (c & 1)];
  }
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
  if (sc) {  // Q8: value scales fold into the probabilities
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[nt][c] *= sc[16 + nt * 8 + tq + (c & 1)];
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
    ldsm_x4_t(vs + swz<D>(tok, d), b0, b1, b2, b3);
    mma_bf16(o[2 * d2], pa, b0, b1);
    mma_bf16(o[2 * d2 + 1], pa, b2, b3);
  }
}

// Transposed form for a private CTA (one sequence, group <= 8 query heads): Sᵀ = K Qᵀ with the 16
// tokens of a block as the MMA rows and the (padded) heads as its 8 columns, then Oᵀ += Vᵀ Pᵀ with
// 16 head dims per MMA row block: D/8 MMAs per block instead of D/4 when the MMA rows held the heads.
// qb: B fragments of Qᵀ (k = dims, n = heads); o: Oᵀ accumulators (rows = dims, cols = heads);
// m, l: running max / sum of heads 2t and 2t+1 (t = lane % 4).
template <int D>
__device__ __forceinline__ void scores_t(const uint32_t (&qb)[D / 16][2], uint32_t ks, float (&s)[4], int lane) {
  s[0] = s[1] = s[2] = s[3] = 0.f;
  const int arow = lane & 15, acol = (lane >> 4) * 8;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a[4];
    ldsm_x4(ks + swz<D>(arow, kk * 16 + acol), a[0], a[1], a[2], a[3]);
    mma_bf16(s, a, qb[kk][0], qb[kk][1]);
  }
}

// Q8 form of scores_t: K straight from the stage's int8 tile (kt). ldmatrix hands lane (g, t) four
// consecutive codes of rows g and g + 8 per 16-byte slice; converted to f16 they fill the MMA's k slots
// 2t, 2t+1, 2t+8, 2t+9 with dims 4t .. 4t+3 of each 16-dim slice, and the query fragments (load_qt8) are
// laid out in the same order, so the dot products are unchanged.
template <int D>
__device__ __forceinline__ void scores_t8(const uint32_t (&qb)[D / 16][2], uint32_t kt, float (&s)[4], int lane) {
  s[0] = s[1] = s[2] = s[3] = 0.f;
  const int row = (lane & 7) + ((lane >> 3) & 1) * 8, half = lane >> 4;
#pragma unroll
  for (int j = 0; j < D / 32; ++j) {
    uint32_t r0, r1, r2, r3;
    ldsm_x4(kt + k8_off<D>(row, 32 * j + 16 * half), r0, r1, r2, r3);
    uint32_t a[4], b[4];
    i8x4_to_f16x4(r0, a[0], a[2]);
    i8x4_to_f16x4(r1, a[1], a[3]);
    mma_f16(s, a, qb[2 * j][0], qb[2 * j][1]);
    i8x4_to_f16x4(r2, b[0], b[2]);
    i8x4_to_f16x4(r3, b[1], b[3]);
    mma_f16(s, b, qb[2 * j + 1][0], qb[2 * j + 1][1]);
  }
}

// Online softmax and Oᵀ += Vᵀ Pᵀ for a tile whose scores Sᵀ (scores_t / scores_t8) are in s.
template <int D>
__device__ __forceinline__ void softmax_pv_t(float (&s)[4], uint32_t vs, int valid, float (&o)[D / 16][4],
                                             float (&m)[2], float (&l)[2], int lane, const float* sc) {
  const int g = lane >> 2, t = lane & 3;
  if (sc) {  // Q8: key scales (rows g and g + 8 are keys)
    const float k0 = sc[g], k1 = sc[g + 8];
    s[0] *= k0;
    s[1] *= k0;
    s[2] *= k1;
    s[3] *= k1;
  }
  if (g >= valid) s[0] = s[1] = -INFINITY;
  if (g + 8 >= valid) s[2] = s[3] = -INFINITY;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float mx = fmaxf(s[r], s[2 + r]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float mn = fmaxf(m[r], mx);
    const float alpha = exp2f(m[r] - mn);
    s[r] = exp2f(s[r] - mn);
    s[2 + r] = exp2f(s[2 + r] - mn);
    float sum = s[r] + s[2 + r];
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    sum += __shfl_xor_sync(0xffffffffu, sum, 8);
    sum += __shfl_xor_sync(0xffffffffu, sum, 16);
    l[r] = l[r] * alpha + sum;
    m[r] = mn;
#pragma unroll
    for (int dt = 0; dt < D / 16; ++dt) {
      o[dt][r] *= alpha;
      o[dt][2 + r] *= alpha;
    }
  }
  // Pᵀ as the B operand (k = tokens, n = heads): thread (g, t) needs tokens 2t, 2t+1, 2t+8, 2t+9 of
  // head g, held (as halves of packed head pairs) by the threads of rows 2t and 2t+1.
  if (sc) {  // Q8: value scales fold into the probabilities
    const float v0 = sc[16 + g], v1 = sc[16 + g + 8];
    s[0] *= v0;
    s[1] *= v0;
    s[2] *= v1;
    s[3] *= v1;
  }
  const uint32_t lo = pack_bf16x2(s[0], s[1]), hi = pack_bf16x2(s[2], s[3]);
  const int src = 8 * t + (g >> 1);
  const uint32_t x = __shfl_sync(0xffffffffu, lo, src), y = __shfl_sync(0xffffffffu, lo, src + 4);
  const uint32_t z = __shfl_sync(0xffffffffu, hi, src), w = __shfl_sync(0xffffffffu, hi, src + 4);
  const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
  const uint32_t b0 = __byte_perm(x, y, sel), b1 = __byte_perm(z, w, sel);
  const int vtok = (lane & 7) + ((lane >> 4) << 3), vdim = ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int dt = 0; dt < D / 16; ++dt) {
    uint32_t a[4];
    ldsm_x4_t(vs + swz<D>(vtok, dt * 16 + vdim), a[0], a[1], a[2], a[3]);
    mma_bf16(o[dt], a, b0, b1);
  }
}

// Q8: probabilities enter the PV MMA in f16, times the value scale and this power of two so that small
// ones stay normal; l carries the same factor, removed before a CTA's partial state leaves it.
constexpr float kPScale = 256.f;

// Q8 form of softmax_pv_t: V straight from the stage's int8 tile (vt, swizzled like K; sc: the stage's 16 K
// then 16 V scales). ldmatrix.trans of the codes as 16-bit pairs hands lane (g, t) the codes of tokens 2t and
// 2t + 1 at dims 2g and 2g + 1 of a 16-dim slice (and tokens 2t + 8, 2t + 9 from the second matrix); split by
// byte they are exactly the A fragment of Vᵀ with MMA row g holding dim 2g and row g + 8 dim 2g + 1 — the
// Oᵀ accumulators keep that order. Value scales of slots past `valid` are taken as 0.
template <int D>
__device__ __forceinline__ void softmax_pv_t8(float (&s)[4], uint32_t vt, const float* sc, int valid,
                                              float (&o)[D / 16][4], float (&m)[2], float (&l)[2], int lane) {
  const int g = lane >> 2, t = lane & 3;
  {
    const float k0 = sc[g], k1 = sc[g + 8];
    s[0] *= k0;
    s[1] *= k0;
    s[2] *= k1;
    s[3] *= k1;
  }
  if (g >= valid) s[0] = s[1] = -INFINITY;
  if (g + 8 >= valid) s[2] = s[3] = -INFINITY;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float mx = fmaxf(s[r], s[2 + r]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float mn = fmaxf(m[r], mx);
    const float alpha = exp2f(m[r] - mn);
    s[r] = exp2f(s[r] - mn);
    s[2 + r] = exp2f(s[2 + r] - mn);
    float sum = s[r] + s[2 + r];
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    sum += __shfl_xor_sync(0xffffffffu, sum, 8);
    sum += __shfl_xor_sync(0xffffffffu, sum, 16);
    l[r] = l[r] * alpha + sum * kPScale;
    m[r] = mn;
#pragma unroll
    for (int dt = 0; dt < D / 16; ++dt) {
      o[dt][r] *= alpha;
      o[dt][2 + r] *= alpha;
    }
  }
  const float v0 = g < valid ? sc[16 + g] * kPScale : 0.f, v1 = g + 8 < valid ? sc[24 + g] * kPScale : 0.f;
  s[0] *= v0;
  s[1] *= v0;
  s[2] *= v1;
  s[3] *= v1;
  const uint32_t lo = pack_f16x2(s[0], s[1]), hi = pack_f16x2(s[2], s[3]);
  const int src = 8 * t + (g >> 1);
  const uint32_t x = __shfl_sync(0xffffffffu, lo, src), y = __shfl_sync(0xffffffffu, lo, src + 4);
  const uint32_t z = __shfl_sync(0xffffffffu, hi, src), w = __shfl_sync(0xffffffffu, hi, src + 4);
  const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
  const uint32_t b0 = __byte_perm(x, y, sel), b1 = __byte_perm(z, w, sel);
  const int row = (lane & 7) + ((lane >> 3) & 1) * 8, half = lane >> 4;
#pragma unroll
  for (int j = 0; j < D / 32; ++j) {
    uint32_t r0, r1, r2, r3;
    ldsm_x4_t(vt + k8_off<D>(row, 32 * j + 16 * half), r0, r1, r2, r3);
    uint32_t a[4];
    i8pairs_to_f16(r0, a[0], a[1]);
    i8pairs_to_f16(r1, a[2], a[3]);
    mma_f16(o[2 * j], a, b0, b1);
    i8pairs_to_f16(r2, a[0], a[1]);
    i8pairs_to_f16(r3, a[2], a[3]);
    mma_f16(o[2 * j + 1], a, b0, b1);
  }
}

template <int D>
__device__ __forceinline__ void attend_tile_t(const uint32_t (&qb)[D / 16][2], uint32_t ks, uint32_t vs, int valid,
                                              float (&o)[D / 16][4], float (&m)[2], float (&l)[2], int lane,
                                              const float* sc = nullptr) {
  float s[4];
  scores_t<D>(qb, ks, s, lane);
  softmax_pv_t<D>(s, vs, valid, o, m, l, lane, sc);
}

// Q8 query fragments for scores_t8 (f16): slot pairs (2t, 2t+1) and (2t+8, 2t+9) of each 16-dim slice
// hold dims 4t, 4t+1 and 4t+2, 4t+3 of it.
template <int D>
__device__ __forceinline__ void load_qt8(uint32_t (&qb)[D / 16][2], const float* qh0, int group, float qscale,
                                         int lane) {
  const int g = lane >> 2, t = lane & 3;
  const float* qh = g < group ? qh0 + g * D : nullptr;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int base = (kk >> 1) * 32 + (kk & 1) * 16 + 4 * t;
    const float4 v = qh ? *reinterpret_cast<const float4*>(qh + base) : make_float4(0.f, 0.f, 0.f, 0.f);
    qb[kk][0] = pack_f16x2(v.x * qscale, v.y * qscale);
    qb[kk][1] = pack_f16x2(v.z * qscale, v.w * qscale);
  }
}

// B fragments of Qᵀ for the transposed form: column n = head g (< group, else zero) of the sequence.
template <int D>
__device__ __forceinline__ void load_qt(uint32_t (&qb)[D / 16][2], const float* qh0, int group, float qscale,
                                        int lane) {
  const int g = lane >> 2, t = lane & 3;
  const float* qh = g < group ? qh0 + g * D : nullptr;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int d0 = kk * 16 + 2 * t;
    const float2 a = qh ? *reinterpret_cast<const float2*>(qh + d0) : make_float2(0.f, 0.f);
    const float2 b = qh ? *reinterpret_cast<const float2*>(qh + d0 + 8) : make_float2(0.f, 0.f);
    qb[kk][0] = pack_bf16x2(a.x * qscale, a.y * qscale);
    qb[kk][1] = pack_bf16x2(b.x * qscale, b.y * qscale);
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
  int64_t num_blocks;
  const int32_t* tables;
  int max_blocks;
  const int32_t* ctx;
  int b, hq, hkv, group;
  int n_shared;   // shared-prefix blocks
  int n_shared_ctas_per_head;
  int n_row_groups;  // shared CTAs per (kv head, chunk): groups of kCons query row tiles
  int nsplit, bps;  // private splits and blocks per split
  int nslots;       // workspace slots per (seq, head) = shared chunks + nsplit
  float qscale;
  __nv_bfloat16* out;
  float* ws_o;  // [b, hq, nslots, d]
  float* ws_ml; // [b, hq, nslots, 2]
  bool direct;  // private CTA writes the final output
  const float* k_scales;  // Q8: fp32 [num_blocks * hkv * 16]
  const float* v_scales;
};

template <int D, bool T, bool Q8>
__device__ void private_cta(const AttnParams& p, const CUtensorMap* tk, const CUtensorMap* tv, int pair, int sp,
                            uint8_t* smem, uint64_t* full, uint64_t* empty) {
  using C = AttnCfg<D, Q8>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = pair / p.hkv, h = pair % p.hkv;
  const int b0 = p.n_shared + sp * p.bps;
  const int32_t* table = p.tables + (int64_t)seq * p.max_blocks;
  const int ctx = p.ctx[seq];
  const int nblk = (ctx + 15) >> 4;
  const bool tables_ok = ctx >= 1 && nblk <= p.max_blocks;
  if (!tables_ok && threadIdx.x == 0) mg_record_error(MG_ERR_DEVICE, 400);
  const int ntiles = tables_ok ? max(0, min(nblk, b0 + p.bps) - b0) : 0;
  const int g0 = lane >> 2, g1 = g0 + 8;
  constexpr int kO = T ? D / 16 : D / 8;  // accumulator fragments: Oᵀ (T) or O
  float o[kO][4];
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < kO; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  if (warp == kProd) {
    // Shared-prefix blocks are read from sequence 0's table: one CTA per sequence checks that its
    // leading entries are the same blocks and records MG_ERR_DEVICE (site 403) when they are not.
    if (p.n_shared > 0 && seq > 0 && h == 0 && sp == 0) {
      bool same = true;
      for (int i = lane; i < p.n_shared; i += 32) same &= table[i] == p.tables[i];
      if (!__all_sync(0xffffffffu, same) && lane == 0) mg_record_error(MG_ERR_DEVICE, 403);
    }
    // Block-table entries 32 at a time, one per lane, the next window loaded a window ahead.
    auto entry = [&](int i) { return i < ntiles ? table[b0 + i] : 0; };
    int cur = entry(lane), nxt = entry(32 + lane);
    bool ok = true;
    for (int i = 0; i < ntiles && ok; ++i) {
      if (i > 0 && (i & 31) == 0) {
        cur = nxt;
        nxt = entry(i + 32 + lane);
      }
      int64_t phys = __shfl_sync(0xffffffffu, cur, i & 31);
      if (phys < 0 || phys >= p.num_blocks) {
        if (lane == 0) mg_record_error(MG_ERR_DEVICE, 401);
        phys = 0;
      }
      if (lane == 0) {
        const int s = i % kStages;
        if (i >= kStages) ok = mbar_wait(&empty[s], ((i / kStages) - 1) & 1, 411);
        if (ok)
          load_stage<D, Q8>(smem, s, tk, tv, &full[s], (int)((phys * p.hkv + h) * 16), p.k_scales, p.v_scales);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
  } else {
    uint32_t qa[D / 16][T ? 2 : 4];
    if constexpr (T && Q8) {
      load_qt8<D>(qa, p.q + ((int64_t)seq * p.hq + h * p.group) * D, p.group, p.qscale, lane);
    } else if constexpr (T) {
      load_qt<D>(qa, p.q + ((int64_t)seq * p.hq + h * p.group) * D, p.group, p.qscale, lane);
    } else {
      load_q<D>(qa, p.q, p.hq, g0 < p.group ? seq : -1, h * p.group + g0, g1 < p.group ? seq : -1,
                h * p.group + g1, p.qscale, lane);
    }
    for (int i = warp; i < ntiles; i += kCons) {
      const int s = i % kStages;
      if (!mbar_wait(&full[s], (i / kStages) & 1, 410)) break;
      const int valid = min(16, ctx - (b0 + i) * 16);
      if constexpr (Q8 && T) {
        // K and V codes go from the stage straight into f16 MMA fragments; the stage is released once the
        // PV MMAs have consumed them
        float sct[4];
        scores_t8<D>(qa, smem_u32(smem + s * C::kTileBytes), sct, lane);
        softmax_pv_t8<D>(sct, smem_u32(smem + C::kVRing + s * C::kTileBytes),
                         reinterpret_cast<const float*>(smem + C::kSRing + s * 128), valid, o, m, l, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      } else if constexpr (Q8) {
        // the stage's codes become this warp's bf16 tiles; the stage is released once they are stored
        uint8_t* wb = smem + C::kBufOffset + warp * C::kBufBytes;
        convert_stage<D>(smem, s, wb, valid, lane, 32, true);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        const uint32_t ks = smem_u32(wb), vs = ks + C::kBf16Tile;
        attend_tile<D>(qa, ks, vs, valid, o, m, l, lane, reinterpret_cast<const float*>(wb + 2 * C::kBf16Tile));
        __syncwarp();  // every lane is done with the buffer before the next conversion
      } else {
        const uint32_t ks = smem_u32(smem + s * C::kStageBytes), vs = ks + C::kTileBytes;
        if (valid < 16) zero_v_tail<D>(vs, valid, lane);
        if constexpr (T) {
          attend_tile_t<D>(qa, ks, vs, valid, o, m, l, lane);
        } else {
          attend_tile<D>(qa, ks, vs, valid, o, m, l, lane);
        }
        if (valid < 16) fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
  }
  __syncthreads();  // every tile consumed: the ring is free for the merge

  // merge the consumer warps' states through shared memory: [warp][row][D + 2]
  float* mg = reinterpret_cast<float*>(smem);
  const int c = (lane & 3) * 2;
  if (T && warp < kCons) {
    // Oᵀ fragment (dims dt*16 + g0 (+8); Q8: dt*16 + 2g0 (+1)), heads c, c+1) -> rows = heads
    constexpr float kUnscale = Q8 ? 1.f / kPScale : 1.f;  // exact: a power of two
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float* dst = mg + (warp * 16 + c + r) * (D + 2);
#pragma unroll
      for (int dt = 0; dt < kO; ++dt) {
        if constexpr (Q8) {
          dst[dt * 16 + 2 * g0] = o[dt][r] * kUnscale;
          dst[dt * 16 + 2 * g0 + 1] = o[dt][2 + r] * kUnscale;
        } else {
          dst[dt * 16 + g0] = o[dt][r];
          dst[dt * 16 + g0 + 8] = o[dt][2 + r];
        }
      }
      if (g0 == 0) {
        dst[D] = m[r];
        dst[D + 1] = l[r] * kUnscale;
      }
    }
  } else if (warp < kCons) {
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
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.group * D; idx += kThreads) {
    const int row = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kCons; ++w) M = fmaxf(M, mg[(w * 16 + row) * (D + 2) + D]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kCons; ++w) {
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

template <int D, bool Q8>
__device__ void shared_cta(const AttnParams& p, const CUtensorMap* tk, const CUtensorMap* tv, int h, int chunk,
                           int rg, uint8_t* smem, uint64_t* full) {
  using C = AttnCfg<D, Q8>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk0 = chunk * kChunk;
  const int nb = min(kChunk, p.n_shared - blk0);
  // shared blocks are the first n_shared entries of every table; read them from sequence 0's table
  if (warp == kProd) {
    int64_t phys = lane < nb ? p.tables[blk0 + lane] : 0;
    if (phys < 0 || phys >= p.num_blocks) {
      mg_record_error(MG_ERR_DEVICE, 402);
      phys = 0;
    }
    for (int i = 0; i < nb; ++i) {
      const int64_t ph = __shfl_sync(0xffffffffu, phys, i);
      if (lane == 0)
        load_stage<D, Q8>(smem, i, tk, tv, &full[i], (int)((ph * p.hkv + h) * 16), p.k_scales, p.v_scales);
    }
    return;
  }
  const int rows = p.b * p.group;
  const int t = rg * kCons + warp;  // this warp's 16-row query tile
  // Q8: every consumer warp converts its share of each stage, so warps without a row tile stay
  if (t * 16 >= rows && !Q8) return;
  const int c = (lane & 3) * 2;
  const int r0 = t * 16 + (lane >> 2), r1 = r0 + 8;
  const int s0 = r0 < rows ? r0 / p.group : -1, s1 = r1 < rows ? r1 / p.group : -1;
  uint32_t qa[D / 16][4];
  load_q<D>(qa, p.q, p.hq, s0, h * p.group + (r0 % p.group), s1, h * p.group + (r1 % p.group), p.qscale, lane);
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  if constexpr (Q8) {
    // Stage i is converted by all consumer warps into buffer i % 2, then each warp runs its rows against
    // it. One consumer barrier per stage: a warp past the barrier of stage i + 1 has finished stage i, so
    // buffer i % 2 is free again when stage i + 2 is converted. Every warp takes every barrier, also after
    // a timed-out wait (the slot is then reported empty).
    bool bad = false;
    for (int i = 0; i < nb; ++i) {
      const bool ok = mbar_wait(&full[i], 0, 412);
      bad |= !ok;
      uint8_t* buf = smem + C::kBufOffset + (i & 1) * C::kBufBytes;
      if (ok) convert_stage<D>(smem, i, buf, 16, threadIdx.x, kCons * 32, true);
      asm volatile("bar.sync 1, %0;" ::"n"(kCons * 32) : "memory");
      if (!bad && t * 16 < rows) {
        const uint32_t ks = smem_u32(buf);
        attend_tile<D>(qa, ks, ks + C::kBf16Tile, 16, o, m, l, lane,
                       reinterpret_cast<const float*>(buf + 2 * C::kBf16Tile));
      }
    }
    if (t * 16 >= rows) return;
    if (bad) {
      m[0] = m[1] = -INFINITY;
      l[0] = l[1] = 0.f;
    }
  } else {
    for (int i = 0; i < nb; ++i) {
      if (!mbar_wait(&full[i], 0, 412)) {
        // timed out (MG_ERR_TIMEOUT recorded): leave an empty state so the merge gives this slot no weight
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
        break;
      }
      const uint32_t ks = smem_u32(smem + i * C::kStageBytes);
      attend_tile<D>(qa, ks, ks + C::kTileBytes, 16, o, m, l, lane);
    }
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

template <int D, bool T, bool Q8>
__global__ void __launch_bounds__(kThreads, 3) paged_attn_kernel(const __grid_constant__ CUtensorMap tk,
                                                              const __grid_constant__ CUtensorMap tv,
                                                              const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + AttnCfg<D, Q8>::kBarOffset);
  uint64_t* empty = full + kStages;
  griddep_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  if (threadIdx.x == kProd * 32) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  __syncthreads();
  griddep_wait();
  const int n_shared_ctas = p.n_shared_ctas_per_head * p.n_row_groups * p.hkv;
  if ((int)blockIdx.x < n_shared_ctas) {
    const int per_head = p.n_shared_ctas_per_head * p.n_row_groups;
    const int h = blockIdx.x / per_head, r = blockIdx.x % per_head;
    shared_cta<D, Q8>(p, &tk, &tv, h, r / p.n_row_groups, r % p.n_row_groups, smem, full);
  } else {
    const int i = blockIdx.x - n_shared_ctas;
    private_cta<D, T, Q8>(p, &tk, &tv, i / p.nsplit, i % p.nsplit, smem, full, empty);
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
  const float* wo = ws_o + sh * nslots * D + d;
  // Slots are read eight at a time with every load of a group issued before any is used, so a merge of
  // n slots waits on about n / 4 memory round trips rather than 2n; the sums keep slot order.
  constexpr int kG = 8;
  float M = -INFINITY;
  for (int s0 = 0; s0 < nslots; s0 += kG) {
    float mv[kG];
#pragma unroll
    for (int j = 0; j < kG; ++j) mv[j] = s0 + j < nslots ? ml[2 * (s0 + j)] : -INFINITY;
#pragma unroll
    for (int j = 0; j < kG; ++j) M = fmaxf(M, mv[j]);
  }
  float L = 0.f, O = 0.f;
  for (int s0 = 0; s0 < nslots; s0 += kG) {
    float mv[kG], lv[kG], ov[kG];
#pragma unroll
    for (int j = 0; j < kG; ++j) {
      const bool in = s0 + j < nslots;
      mv[j] = in ? ml[2 * (s0 + j)] : -INFINITY;
      lv[j] = in ? ml[2 * (s0 + j) + 1] : 0.f;
      ov[j] = in ? wo[(int64_t)(s0 + j) * D] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kG; ++j) {
      if (s0 + j < nslots) {
        const float w = M == -INFINITY ? 0.f : exp2f(mv[j] - M);
        L += lv[j] * w;
        O += ov[j] * w;
      }
    }
  }
  out[sh * D + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
}

struct Plan {
  int n_shared_ctas_per_head, n_row_groups, nsplit, bps, nslots;
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

// Splits: private CTAs for about two and a half waves of three CTAs per SM beside the shared CTAs
// (small enough that the last wave's tail is short), with at least two tiles per consumer warp.
Plan make_plan(int b, int hq, int hkv, int d, int max_blocks, int n_shared) {
  Plan pl{};
  pl.n_shared_ctas_per_head = (n_shared + kChunk - 1) / kChunk;
  const int row_tiles = (b * (hq / hkv) + 15) / 16;
  pl.n_row_groups = (row_tiles + kCons - 1) / kCons;
  const int priv_max = max_blocks - n_shared > 0 ? max_blocks - n_shared : 1;
  const int pairs = b * hkv;
  const int target = 15 * sm_count_attn() / 2 - pl.n_shared_ctas_per_head * pl.n_row_groups * hkv;
  int nsplit = target > pairs ? (target + pairs - 1) / pairs : 1;
  const int max_split = (priv_max + 2 * kCons - 1) / (2 * kCons);
  nsplit = nsplit > max_split ? max_split : nsplit;
  nsplit = nsplit < 1 ? 1 : nsplit;
  pl.bps = (priv_max + nsplit - 1) / nsplit;
  pl.nsplit = (priv_max + pl.bps - 1) / pl.bps;
  pl.nslots = pl.n_shared_ctas_per_head + pl.nsplit;
  pl.direct = pl.nslots == 1;
  pl.ws_bytes = pl.direct ? 0 : (size_t)b * hq * pl.nslots * (size_t)(d + 2) * sizeof(float);
  return pl;
}

template <int D, bool Q8 = false>
int launch_attn(AttnParams& p, const Plan& pl, const void* k_pool, const void* v_pool, cudaStream_t st) {
  using C = AttnCfg<D, Q8>;
  static bool attr_done[64] = {};
  static std::mutex attr_mu;
  MG_CUDA_TRY(mg_once_per_device(attr_done, attr_mu, [] {
    cudaError_t e = cudaFuncSetAttribute(paged_attn_kernel<D, true, Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(paged_attn_kernel<D, false, Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C::kSmem);
    return e;
  }));
  // Pools as 2-D tensors [num_blocks*hkv*16 rows, D]: rows of one (block, kv head) tile are adjacent.
  const uint64_t rows = (uint64_t)p.num_blocks * p.hkv * 16;
  if (rows > 0x7fffffffull) return MG_ERR_UNSUPPORTED;
  CUtensorMap tk, tv;
  int rc;
  if constexpr (Q8) {  // int8 rows of d bytes, one box per tile, swizzled for the consumers' ldmatrix reads
    const CUtensorMapSwizzle ksw = D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                            : (D == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    rc = mg_make_map_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_pool, D, rows, D, D, 16, ksw);
    if (rc) return rc;
    rc = mg_make_map_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, v_pool, D, rows, D, D, 16, ksw);
  } else {
    const CUtensorMapSwizzle sw = D >= 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    rc = mg_make_map_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k_pool, D, rows, D * 2, C::kBoxCols, 16, sw);
    if (rc) return rc;
    rc = mg_make_map_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, v_pool, D, rows, D * 2, C::kBoxCols, 16, sw);
  }
  if (rc) return rc;
  p.n_shared_ctas_per_head = pl.n_shared_ctas_per_head;
  p.n_row_groups = pl.n_row_groups;
  const int64_t ctas = (int64_t)pl.n_shared_ctas_per_head * pl.n_row_groups * p.hkv +
                       (int64_t)p.b * p.hkv * pl.nsplit;
  if (ctas > 0x7fffffff) return MG_ERR_UNSUPPORTED;
  if (p.group <= 8) {
    MG_CUDA_TRY(mg_launch(paged_attn_kernel<D, true, Q8>, dim3((unsigned)ctas), dim3(kThreads), C::kSmem, st, 1, tk,
                          tv, p));
  } else {
    MG_CUDA_TRY(mg_launch(paged_attn_kernel<D, false, Q8>, dim3((unsigned)ctas), dim3(kThreads), C::kSmem, st, 1, tk,
                          tv, p));
  }
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

namespace {

int paged_attn(const float* q, const void* k_pool, const void* v_pool, const float* k_scales, const float* v_scales,
               bool q8, int64_t num_blocks, const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens,
               int b, int hq, int hkv, int d, int n_shared_blocks, float scale, void* out, void* workspace,
               size_t workspace_bytes, void* stream) {
  if (b < 0 || hq <= 0 || hkv <= 0 || hq % hkv || hq / hkv > 16 || max_blocks <= 0 || num_blocks <= 0 ||
      n_shared_blocks < 0 || n_shared_blocks > max_blocks || !q || !k_pool || !v_pool || !block_tables ||
      !ctx_lens || !out || (q8 && (!k_scales || !v_scales)))
    return MG_ERR_INVALID_ARG;
  if (d != 32 && d != 64 && d != 128) return MG_ERR_UNSUPPORTED;
  if (b == 0) return MG_OK;
  const Plan pl = make_plan(b, hq, hkv, d, max_blocks, n_shared_blocks);
  if (pl.ws_bytes > 0 && (!workspace || workspace_bytes < pl.ws_bytes)) return MG_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) | reinterpret_cast<uintptr_t>(q) |
       reinterpret_cast<uintptr_t>(k_scales) | reinterpret_cast<uintptr_t>(v_scales)) & 15)
    return MG_ERR_INVALID_ARG;
  AttnParams p{};
  p.q = q;
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
  p.k_scales = k_scales;
  p.v_scales = v_scales;
  cudaStream_t st = mg_stream(stream);
  if (q8) {
    if (d == 32) return launch_attn<32, true>(p, pl, k_pool, v_pool, st);
    return d == 64 ? launch_attn<64, true>(p, pl, k_pool, v_pool, st) : launch_attn<128, true>(p, pl, k_pool, v_pool, st);
  }
  if (d == 32) return launch_attn<32>(p, pl, k_pool, v_pool, st);
  return d == 64 ? launch_attn<64>(p, pl, k_pool, v_pool, st) : launch_attn<128>(p, pl, k_pool, v_pool, st);
}

}  // namespace

extern "C" int mg_paged_decode_attn(const float* q, const void* k_pool, const void* v_pool, int64_t num_blocks,
                                    const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens, int b,
                                    int hq, int hkv, int d, int n_shared_blocks, float scale, void* out,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  return paged_attn(q, k_pool, v_pool, nullptr, nullptr, false, num_blocks, block_tables, max_blocks, ctx_lens, b,
                    hq, hkv, d, n_shared_blocks, scale, out, workspace, workspace_bytes, stream);
}

extern "C" int mg_paged_decode_attn_kv8(const float* q, const int8_t* k_pool, const int8_t* v_pool,
                                        const float* k_scales, const float* v_scales, int64_t num_blocks,
                                        const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens, int b,
                                        int hq, int hkv, int d, int n_shared_blocks, float scale, void* out,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  return paged_attn(q, k_pool, v_pool, k_scales, v_scales, true, num_blocks, block_tables, max_blocks, ctx_lens, b,
                    hq, hkv, d, n_shared_blocks, scale, out, workspace, workspace_bytes, stream);
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
