// Persistent decode-layer kernel: everything of a decoder layer that sits between two paged
// attentions, in ONE launch —
//
//   O-proj (+bias, +residual | peer push)  -> norm (post-attention)  -> gate/up (SwiGLU | GELU)
//   -> down (+bias, +residual | peer push)  -> norm (next layer's input norm, or the final norm)
//   -> QKV (+bias) with RoPE and the paged K/V append of the next layer
//
// Why: a decode step at batch <= 32 streams ~100 MB of INT8 weights per layer through four skinny
// linears. As separate kernels every boundary drains the HBM pipe (dependency release, first
// activation tile, split-K reduction, wave tail). Here one CTA per SM streams its share of ALL four
// weight matrices through a deep shared-memory ring without ever stopping: weights never depend on
// activations, so the TMA producer runs ahead across phase boundaries while the phases' data
// dependencies are carried by counters in global memory instead of kernel boundaries.
//
// Work split. Each linear's work is its list of units (128-row weight tile t, 128-column K block
// kb), u = t*KB + kb — the order of the tile-packed codes in memory. CTA c of G takes the contiguous
// units [U*c/G, U*(c+1)/G) of every linear (stream-K): equal weight bytes per SM, no wave tail. A
// CTA's run inside one tile is a segment; its fp32 partial goes to a workspace slot and the segment
// counts its K blocks into the tile's ticket. The CTA that completes the ticket finishes the tile:
// it adds the tile's partials in slot order (the sum does not depend on timing: bit-reproducible)
// and applies the epilogue (scale, bias, residual add, SwiGLU / GELU, RoPE + K/V append).
//
// Warp roles (15 warps):
//   warp 8        weight producer (one thread): TMA loads of the weight tiles into a ring of kSW 16 KB
//                 stages, from the first instruction on (weights depend on nothing);
//   warp 14       activation producer (one thread): TMA loads of the [MP x 128] bf16 activation tile of each
//                 unit into a ring of kSX stages once the phase's input is final;
//   warps 0..7    converters: int8 weight bytes -> exact bf16 in a TMEM ring of A operands;
//   warp 9        MMA issuer: tcgen05.mma kind::f16 (A from TMEM, B = activations in shared memory)
//                 into one of two TMEM accumulators (swap-AB: weight rows = MMA M, tokens = MMA N);
//   warps 10..13  epilogue: drain accumulators, tickets, tile finishing, and the norm rows.
// Norms: CTA c < m normalises token row c once every tile that feeds it is final (a counter), then
// counts itself in; the next linear's producer waits for all m rows.
//
// Tensor parallelism: the O and down tiles are partial sums. A finisher pushes its tile (scale
// applied, bias not) into every rank's receive area as tagged 64-bit words {bf16 v[n], bf16 v[n+1],
// epoch} — the protocol of the separate row-parallel kernels (comm.cu) — and the norm row sums the
// world partials in rank order onto the residual (identical bits on every rank), adds the bias once,
// then normalises.
//
// Every wait is bounded (globaltimer deadline, or an error already recorded in the device error word):
// a wait that gives up records MG_ERR_TIMEOUT and the CTA unwinds.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

constexpr int kBN = 128;
constexpr int kBK = 128;
constexpr int kConvWarps = 8;
constexpr int kProdWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kEpiWarp0 = 10;
constexpr int kEpiWarps = 4;
constexpr int kXWarp = 14;                               // activation loader
constexpr int kThreads = (kXWarp + 1) * 32;             // 480
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr uint32_t kWBytes = kBN * kBK;  // one int8 weight tile
constexpr int kMP = 32;                  // tokens per launch (MMA N)

enum { L_O = 0, L_GU = 1, L_DN = 2, L_QKV = 3, kNLin = 4 };
// control words (all zero between launches)
enum { C_EXIT = 0, C_O_DONE = 1, C_N2_DONE = 2, C_GU_DONE = 3, C_DN_DONE = 4, C_N1_DONE = 5, C_HDR = 8 };

struct BlkCfg {
  static constexpr int kSW = 7;   // weight stages
  static constexpr int kSX = 12;  // activation stages
  static constexpr int kNA = 3;   // bf16 A tiles in TMEM (64 columns each)
  static constexpr uint32_t kXBytes = kMP * kBK * 2;
  static constexpr uint32_t kXOff = kSW * kWBytes;
  static constexpr uint32_t kStgOff = kXOff + kSX * kXBytes;
  static constexpr uint32_t kStgBytes = kMP * kBN * 4;
  static constexpr uint32_t kBarOff = kStgOff + kStgBytes;
  static constexpr uint32_t kSmem = kBarOff + 512 + 1024;
  // Accumulators: 2 buffers, one drains while the next segment accumulates.
  static constexpr uint32_t kAcc0 = kNA * 64;
  static constexpr uint32_t kTmemCols = 256;
  static_assert(kAcc0 + 2 * kMP <= kTmemCols, "TMEM budget");
  // D=fp32, A=B=bf16, K-major, N = kMP, M = 128
  static constexpr uint32_t kIdesc =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kMP >> 3) << 17) | ((uint32_t)(kBN >> 4) << 24);
};

struct Lin {
  const float* scales;
  const float* bias;
  float* part;       // [tiles][maxslots][128 rows][kMP] fp32 partials (a row's tokens contiguous)
  uint32_t* ticket;  // [tiles] K blocks accounted for
  int64_t units;     // tiles * kb
  int tiles, kb, maxslots, k;
};

struct Params {
  int m, flags, hidden, act_cols, nqkv, hq, hkv, d, norm, mlp, G, ctl_words, max_pos, pad;
  float eps;
  Lin lin[kNLin];
  float* h;
  const float *n2_w, *n2_b, *n1_w, *n1_b;
  __nv_bfloat16 *x2, *x1, *act;
  const float* cos_sin;
  const int32_t *positions, *slots;
  float* q_out;
  __nv_bfloat16 *k_pool, *v_pool;
  int64_t num_blocks;
  uint32_t* ctl;
  uint64_t timeout_ns;
  PeerOut po;         // world > 1: row-parallel push / reduce
};

struct Maps {
  CUtensorMap w[kNLin];
  CUtensorMap x[kNLin];
};

__device__ __forceinline__ bool lin_on(const Params& p, int ph) {
  switch (ph) {
    case L_O: return p.flags & MG_BLK_O;
    case L_GU:
    case L_DN: return p.flags & MG_BLK_MLP;
    default: return p.flags & MG_BLK_QKV;
  }
}

// Unit arithmetic is 32-bit (units * G < 2^32: the host caps units * 128 below 2^31 and G at 256); the
// per-unit loops keep their tile / K block incrementally, with no division (a 64-bit division is a long
// software routine on the GPU, and these loops are the kernel's critical path).
__device__ __forceinline__ int rstart(int64_t units, int c, int G) {
  return (int)((uint32_t)units * (uint32_t)c / (uint32_t)G);
}
// CTA owning unit u: the largest c with rstart(c) <= u.
__device__ __forceinline__ int owner(int64_t units, int64_t u, int G) {
  return (int)((((uint32_t)u + 1u) * (uint32_t)G - 1u) / (uint32_t)units);
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// Orders this thread's generic-proxy global accesses with its async-proxy (TMA) accesses: writers of an
// activation another CTA loads by TMA fence after their stores, the loader after its acquire.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Epilogue thread -> weight row of the tile: warp w may only read TMEM lanes 32*(w%4) .. 32*(w%4)+31.
__device__ __forceinline__ int epi_row() { return ((threadIdx.x >> 5) & 3) * 32 + (threadIdx.x & 31); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float gelu_tanh_f(float v) {
  return 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

// Shared-memory descriptor of a K-major, 128B-swizzled bf16 tile (8-row x 128 B atoms, 1024 B apart).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Bounded waits. `abort` (shared) ends every wait of the CTA once one of them gave up; an error
// recorded anywhere on the device ends the waits on other CTAs' counters.
struct Ctx {
  volatile int* abort;
  uint64_t timeout_ns;
  const uint32_t* ctl;
};

// Snapshot of the first wait that gave up on this device (read by mg_decode_block_diag): the site, the
// CTA and thread, two site-specific words (unit / segment / phase), the control words and how many
// gate/up tiles were final.
__device__ uint32_t g_blk_diag[32];
// Progress of every CTA of the latest launch (for the diagnosis above): [cta][role] with role 0 = producer
// (x loads | weight loads << 16), 1 = converters (units), 2 = MMA (units | segments << 16), 3 = epilogue
// (segments | stage << 16; stage 0 O, 1 N2, 2 gate/up, 3 down, 4 N1, 5 QKV, 6 done).
constexpr int kDiagCtas = 256;
__device__ uint32_t g_blk_prog[kDiagCtas][4];
__device__ uint32_t g_blk_snap[kDiagCtas][4];  // g_blk_prog when the first wait gave up
// Timeline of the latest launch: globaltimer (ns) at 16 points per CTA (mg_decode_block_trace).
constexpr int kTracePoints = 16;
__device__ uint64_t g_blk_ts[kDiagCtas][kTracePoints];
__device__ __forceinline__ void trace(int point) {
  if (blockIdx.x < kDiagCtas) g_blk_ts[blockIdx.x][point] = global_ns();
}
__device__ __forceinline__ void prog(int role, uint32_t v) {
  if (blockIdx.x < kDiagCtas) *reinterpret_cast<volatile uint32_t*>(&g_blk_prog[blockIdx.x][role]) = v;
}

__device__ __noinline__ bool fail(const Ctx& x, int where, uint32_t a = 0, uint32_t b = 0) {
  // the snapshot is taken before the error is recorded: other CTAs unwind once they see the error
  if (atomicCAS(&g_blk_diag[0], 0u, (uint32_t)where) == 0u) {
    g_blk_diag[1] = blockIdx.x;
    g_blk_diag[2] = threadIdx.x;
    g_blk_diag[3] = a;
    g_blk_diag[4] = b;
    for (int i = 0; i < 8; ++i) g_blk_diag[8 + i] = x.ctl ? *reinterpret_cast<const volatile uint32_t*>(x.ctl + i) : 0u;
    for (int i = 0; i < kDiagCtas; ++i)
      reinterpret_cast<uint4*>(&g_blk_snap[0][0])[i] = __ldcg(reinterpret_cast<const uint4*>(&g_blk_prog[0][0]) + i);
    __threadfence();
  }
  mg_record_error(MG_ERR_TIMEOUT, where);
  *x.abort = 1;
  return false;
}

__device__ bool mbar_wait_ab(const Ctx& x, uint64_t* bar, uint32_t parity, int where, uint32_t a = 0,
                             uint32_t b = 0) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15) == 15) {
      if (*x.abort) return false;
      const uint64_t t = global_ns();
      if (!t0) t0 = t;
      else if (t - t0 > x.timeout_ns) return fail(x, where, a, b);
    }
  }
}

// Wait until *p >= target (acquire).
__device__ bool wait_ge(const Ctx& x, const uint32_t* p, uint32_t target, int where) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_u32(p) >= target) return true;
    if ((i & 7) == 7) {
      if (*x.abort) return false;
      if (*reinterpret_cast<volatile int*>(&g_mg_dev_error) != 0) {
        *x.abort = 1;
        return false;
      }
      const uint64_t t = global_ns();
      if (!t0) t0 = t;
      else if (t - t0 > x.timeout_ns) return fail(x, where, target, ld_acquire_u32(p));
      __nanosleep(64);
    }
  }
}

// Cursor over this CTA's units of the enabled linears, in phase order.
struct Cur {
  int ph;
  int u, u0, u1;  // unit, this CTA's range [u0, u1) of the phase
  int kb, KB;     // u % KB, kept incrementally
};
__device__ __forceinline__ void cur_next_phase(const Params& p, int c, Cur& k) {
  while (k.ph < kNLin && (k.ph < 0 || !lin_on(p, k.ph) || k.u >= k.u1)) {
    ++k.ph;
    if (k.ph < kNLin && lin_on(p, k.ph)) {
      k.u = k.u0 = rstart(p.lin[k.ph].units, c, p.G);
      k.u1 = rstart(p.lin[k.ph].units, c + 1, p.G);
      k.KB = p.lin[k.ph].kb;
      k.kb = k.u % k.KB;
    }
  }
}
__device__ __forceinline__ Cur cur_begin(const Params& p, int c) {
  Cur k{-1, 0, 0, 0, 0, 1};
  cur_next_phase(p, c, k);
  return k;
}
__device__ __forceinline__ void cur_advance(const Params& p, int c, Cur& k) {
  ++k.u;
  if (++k.kb == k.KB) k.kb = 0;
  if (k.u >= k.u1) cur_next_phase(p, c, k);
}

// Is the activation tile of unit (ph, u) ready to load?
__device__ __forceinline__ bool x_ready(const Params& p, int ph, int64_t u) {
  switch (ph) {
    case L_O: return true;
    case L_GU: return ld_acquire_u32(p.ctl + C_N2_DONE) >= (uint32_t)p.m;
    case L_DN: return ld_acquire_u32(p.ctl + C_GU_DONE) >= (uint32_t)p.lin[L_GU].tiles;
    default: return !(p.flags & MG_BLK_N1) || ld_acquire_u32(p.ctl + C_N1_DONE) >= (uint32_t)p.m;
  }
}

// ---------------------------------------------------------------------------------------------
// Epilogue-warp helpers (128 threads; thread e <-> weight row e of the tile)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float epi_sum(float v, float* red) {
  v = warp_sum(v);
  const int e = epi_row();
  epi_bar();
  if ((e & 31) == 0) red[e >> 5] = v;
  epi_bar();
  return red[0] + red[1] + red[2] + red[3];
}

// The epilogue warps decide together: a failure seen by any of their threads (which set the CTA's
// abort flag) stops all 128 of them at the same point, so every named barrier is reached by all or none.
__device__ __forceinline__ bool epi_stop(volatile int* abort, int* s_stop) {
  const int e = epi_row();
  epi_bar();
  if (e == 0) *s_stop = *abort;
  epi_bar();
  return *reinterpret_cast<volatile int*>(s_stop) != 0;
}

// The norm of token row `row`: with world > 1 first the all-reduce of the preceding row-parallel
// linear (sum of the world partials in rank order + bias onto the residual), then RMSNorm / LayerNorm
// into x (bf16). All 128 epilogue threads.
__device__ bool norm_row(const Params& p, const Ctx& cx, int row, const float* w, const float* wb,
                         const float* rp_bias, uint32_t epoch, __nv_bfloat16* x, float* red, int* s_stop) {
  const int e = epi_row();
  const int H = p.hidden;
  float* hr = p.h + (int64_t)row * H;
  bool ok = true;
  if (epoch) {  // row-parallel reduce: words of this row from every rank
    const PeerOut& po = p.po;
    const uint64_t* base = po.recv[po.rank] + (int64_t)(epoch & 1u) * po.world * po.slot + (int64_t)row * (H / 2);
    uint64_t t0 = 0;
    for (int i = e; i < H / 2; i += kEpiThreads) {
      float a0 = __ldcg(hr + 2 * i), a1 = __ldcg(hr + 2 * i + 1);
      // every rank's word of this pair is loaded before any is used: one round trip for the world
      uint64_t wds[MG_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < MG_MAX_RANKS; ++r)
        if (r < po.world) wds[r] = *reinterpret_cast<const volatile uint64_t*>(base + (int64_t)r * po.slot + i);
#pragma unroll
      for (int r = 0; r < MG_MAX_RANKS && ok; ++r) {
        if (r >= po.world) break;
        const uint64_t* wp = base + (int64_t)r * po.slot + i;
        uint64_t wd = wds[r];
        for (uint32_t spin = 0;; ++spin) {
          if ((uint32_t)(wd >> 32) == epoch) break;
          wd = *reinterpret_cast<const volatile uint64_t*>(wp);
          if ((uint32_t)(wd >> 32) == epoch) break;
          if ((spin & 15) == 15) {
            if (*cx.abort || *reinterpret_cast<volatile int*>(&g_mg_dev_error) != 0) {
              *cx.abort = 1;
              ok = false;
              break;
            }
            const uint64_t t = global_ns();
            if (!t0) t0 = t;
            else if (t - t0 > p.po.timeout_ns) {
              ok = fail(cx, 760 + r);
              break;
            }
          }
        }
        if (!ok) break;
        a0 += bf16lo((uint32_t)wd);
        a1 += bf16hi((uint32_t)wd);
      }
      if (rp_bias) {
        a0 += rp_bias[2 * i];
        a1 += rp_bias[2 * i + 1];
      }
      hr[2 * i] = a0;
      hr[2 * i + 1] = a1;
    }
    __threadfence();
    if (epi_stop(cx.abort, s_stop)) return false;
  }
  float s1 = 0.f;
  for (int i = e; i < H; i += kEpiThreads) {
    const float v = __ldcg(hr + i);
    s1 += p.norm == MG_NORM_LAYER ? v : v * v;
  }
  float mean = 0.f, inv;
  if (p.norm == MG_NORM_LAYER) {
    mean = epi_sum(s1, red) / (float)H;
    epi_bar();  // red reused
    float s2 = 0.f;
    for (int i = e; i < H; i += kEpiThreads) {
      const float v = __ldcg(hr + i) - mean;
      s2 += v * v;
    }
    inv = rsqrtf(epi_sum(s2, red) / (float)H + p.eps);
  } else {
    inv = rsqrtf(epi_sum(s1, red) / (float)H + p.eps);
  }
  __nv_bfloat16* xr = x + (int64_t)row * H;
  for (int i = e; i < H; i += kEpiThreads) {
    const float v = __ldcg(hr + i);
    const float o = p.norm == MG_NORM_LAYER ? (v - mean) * inv * w[i] + wb[i] : w[i] * (v * inv);
    xr[i] = __float2bfloat16_rn(o);
  }
  return ok;  // uniform: a failure returned above, for all threads
}

// Tile finisher: adds the tile's partials in slot order into `stg` ([kMP tokens][128 rows] fp32 shared
// staging), then applies the phase's epilogue from there (epilogues that pair rows read the partner row).
__device__ void finish_tile(const Params& p, const Ctx& cx, int ph, int t, float* stg, uint32_t epoch) {
  const int e = epi_row();
  const Lin& L = p.lin[ph];
  const int G = p.G;
  const int64_t u_first = (int64_t)t * L.kb, u_last = u_first + L.kb - 1;
  const int c_first = owner(L.units, u_first, G), c_last = owner(L.units, u_last, G);
  // This thread's row of every slot is kMP contiguous floats. Half a row (16 tokens = 4 float4) of up to
  // three slots is loaded per round trip (12 loads in flight), and the slots are added in slot order.
  constexpr int kH = kMP / 2, kHQ = kH / 4, kSlotsPerTrip = 3;
  const float4* base = reinterpret_cast<const float4*>(L.part + ((int64_t)t * L.maxslots * kBN + e) * kMP);
  const int64_t slot_q = (int64_t)kBN * (kMP / 4);  // float4 per slot
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float v[kH];
#pragma unroll
    for (int j = 0; j < kH; ++j) v[j] = 0.f;
    for (int c = c_first; c <= c_last; c += kSlotsPerTrip) {
      float4 a[kSlotsPerTrip][kHQ];
      bool ok[kSlotsPerTrip];
#pragma unroll
      for (int k = 0; k < kSlotsPerTrip; ++k) {
        ok[k] = c + k <= c_last && rstart(L.units, c + k, G) < rstart(L.units, c + k + 1, G);  // CTAs without
#pragma unroll                                                                             // units: no partial
        for (int q = 0; q < kHQ; ++q)
          a[k][q] = ok[k] ? __ldcg(base + (c + k - c_first) * slot_q + half * kHQ + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < kSlotsPerTrip; ++k) {
        if (!ok[k]) continue;
#pragma unroll
        for (int q = 0; q < kHQ; ++q) {
          v[4 * q] += a[k][q].x;
          v[4 * q + 1] += a[k][q].y;
          v[4 * q + 2] += a[k][q].z;
          v[4 * q + 3] += a[k][q].w;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kH; ++j) stg[(half * kH + j) * kBN + e] = v[j];
  }
  epi_bar();
  const int64_t n = (int64_t)t * kBN + e;
  if (ph == L_O || ph == L_DN) {
    const float s = L.scales[n];
    if (epoch) {  // row-parallel: push (scale applied, bias added once by the reduce)
      const PeerOut& po = p.po;
      const uint64_t tag = (uint64_t)epoch << 32;
      const int64_t set_off = ((int64_t)(epoch & 1u) * po.world + po.rank) * po.slot;
      for (int j = 0; j < p.m; ++j) {
        const float a = stg[j * kBN + e] * s;
        const float b = __shfl_down_sync(0xffffffffu, a, 1);
        if ((e & 1) == 0) {
          const uint64_t word = tag | pack_bf16x2(a, b);
          const int64_t off = set_off + ((int64_t)j * p.hidden + n) / 2;
          for (int r = 0; r < po.world; ++r) st_volatile_u64(po.recv[r] + off, word);
        }
      }
    } else {
      const float b = L.bias ? L.bias[n] : 0.f;
      for (int j0 = 0; j0 < p.m; j0 += 8) {  // residual reads batched: 8 in flight
        float hv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) hv[k] = j0 + k < p.m ? __ldcg(p.h + (int64_t)(j0 + k) * p.hidden + n) : 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (j0 + k < p.m) p.h[(int64_t)(j0 + k) * p.hidden + n] = hv[k] + (stg[(j0 + k) * kBN + e] * s + b);
      }
    }
    __threadfence();
    epi_bar();  // also: every thread is done with stg
    if (e == 0) atom_add_acq_rel(p.ctl + (ph == L_O ? C_O_DONE : C_DN_DONE), 1u);
    return;
  }
  if (ph == L_GU) {
    if (p.mlp == MG_EPI_SWIGLU_BF16) {
      const int r = e & 63;
      const int64_t ng = (int64_t)t * kBN + r, nu = ng + 64;
      const float sg = L.scales[ng], su = L.scales[nu];
      const float bg = L.bias ? L.bias[ng] : 0.f, bu = L.bias ? L.bias[nu] : 0.f;
      for (int j = e >> 6; j < p.m; j += 2) {
        const float g = stg[j * kBN + r] * sg + bg, u = stg[j * kBN + r + 64] * su + bu;
        p.act[(int64_t)j * p.act_cols + (int64_t)t * 64 + r] = __float2bfloat16_rn(silu_f(g) * u);
      }
    } else {
      const float s = L.scales[n], b = L.bias ? L.bias[n] : 0.f;
      for (int j = 0; j < p.m; ++j)
        p.act[(int64_t)j * p.act_cols + n] = __float2bfloat16_rn(gelu_tanh_f(stg[j * kBN + e] * s + b));
    }
    fence_proxy_async_global();
    __threadfence();
    epi_bar();  // also: every thread is done with stg
    if (e == 0) atom_add_acq_rel(p.ctl + C_GU_DONE, 1u);
    return;
  }
  // QKV: scale + bias, RoPE on q and k, q to q_out (fp32), k / v into the token's paged slot (bf16)
  {
    const bool valid = n < p.nqkv;
    const float s = valid ? L.scales[n] : 0.f, b = (valid && L.bias) ? L.bias[n] : 0.f;
    for (int j = 0; j < p.m; ++j) stg[j * kBN + e] = stg[j * kBN + e] * s + b;  // own column only
    epi_bar();
    if (valid) {
      const int D = p.d, half = D >> 1;
      const int hd = (int)(n / D), dd = (int)(n % D);
      const int partner = dd < half ? e + half : e - half;
      const bool rope = p.cos_sin && hd < p.hq + p.hkv;
      const int jj = dd < half ? dd : dd - half;
      for (int j = 0; j < p.m; ++j) {
        float val = stg[j * kBN + e];
        if (rope) {
          const int pos = p.positions[j];
          if (pos < 0 || pos >= p.max_pos) {
            mg_record_error(MG_ERR_DEVICE, 770);
            continue;
          }
          const float cs = p.cos_sin[(int64_t)pos * D + jj], sn = p.cos_sin[(int64_t)pos * D + half + jj];
          const float pv = stg[j * kBN + partner];
          val = dd < half ? val * cs - pv * sn : val * cs + pv * sn;
        }
        if (hd < p.hq) {
          p.q_out[((int64_t)j * p.hq + hd) * D + dd] = val;
        } else {
          const int slot = p.slots[j];
          const int64_t blk = slot >> 4;
          if (slot < 0 || blk >= p.num_blocks) {
            mg_record_error(MG_ERR_DEVICE, 771);
            continue;
          }
          const bool is_k = hd < p.hq + p.hkv;
          const int kh = is_k ? hd - p.hq : hd - p.hq - p.hkv;
          __nv_bfloat16* dst = (is_k ? p.k_pool : p.v_pool) + ((blk * p.hkv + kh) * 16 + (slot & 15)) * (int64_t)D;
          dst[dd] = __float2bfloat16_rn(val);
        }
      }
    }
    epi_bar();  // stg is reused by the next finish
  }
}

// ---------------------------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) decode_block_kernel(const __grid_constant__ Maps maps, const Params p) {
  using C = BlkCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* wempty = wfull + C::kSW;
  uint64_t* xfull = wempty + C::kSW;
  uint64_t* xempty = xfull + C::kSX;
  uint64_t* afull = xempty + C::kSX;
  uint64_t* aempty = afull + C::kNA;
  uint64_t* accfull = aempty + C::kNA;  // [2]
  uint64_t* accempty = accfull + 2;     // [2]
  uint64_t* mma_fin = accempty + 2;     // every MMA of the CTA has completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_fin + 1);
  float* stg = reinterpret_cast<float*>(smem + C::kStgOff);
  __shared__ volatile int s_abort;
  __shared__ int s_flag, s_stop;
  __shared__ float s_red[kEpiWarps];

  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  if (threadIdx.x == 0) trace(0);
  const Ctx cx{&s_abort, p.timeout_ns, p.ctl};

  if (threadIdx.x == 0) {
    for (int r = 0; r < 4; ++r) prog(r, 0u);
    s_abort = 0;
    for (int s = 0; s < C::kSW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kConvWarps);
    }
    for (int s = 0; s < C::kSX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int b = 0; b < C::kNA; ++b) {
      mbar_init(&afull[b], kConvWarps);
      mbar_init(&aempty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], kEpiWarps);
    }
    mbar_init(mma_fin, 1);
    fence_mbar_init();
  }
  if (warp == kProdWarp && lane == 0) {
    for (int i = 0; i < kNLin; ++i)
      if (lin_on(p, i)) {
        tma_prefetch_desc(&maps.w[i]);
        tma_prefetch_desc(&maps.x[i]);
      }
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == kProdWarp) {
    // ------------------------------- weight producer (TMA) -------------------------------
    // Weights never depend on another kernel or CTA: the ring is kept full from the first instruction.
    if (lane == 0) {
      Cur kw = cur_begin(p, c);
      int iw = 0;
      // weights are read exactly once: evict them from L2 first, so the activations the phases exchange stay
      const uint64_t evict_first = l2_policy_evict_first();
      uint32_t polls = 0;
      uint64_t t0 = 0;
      while (kw.ph < kNLin && !s_abort) {
        if (iw < C::kSW || mbar_test_wait(&wempty[iw % C::kSW], ((iw / C::kSW) - 1) & 1)) {
          const int s = iw % C::kSW;
          mbar_arrive_expect_tx(&wfull[s], kWBytes);
          tma_load_2d_hint(smem + s * kWBytes, &maps.w[kw.ph], &wfull[s], 0, (int)(kw.u * kBN), evict_first);
          ++iw;
          cur_advance(p, c, kw);
          if ((iw & 7) == 0) prog(0, (uint32_t)iw << 16);
          polls = 0;
          t0 = 0;
        } else if ((++polls & 15) == 0) {
          const uint64_t t = global_ns();
          if (!t0) t0 = t;
          else if (t - t0 > p.timeout_ns) {
            fail(cx, 700, (uint32_t)iw, ((uint32_t)(kw.ph & 0xff) << 24) | (uint32_t)kw.u);
            break;
          }
          __nanosleep(32);
        }
      }
      // shared memory is the destination of every load issued: all of them land before the CTA exits
      for (int s = 0; s < C::kSW && s < iw; ++s) mbar_wait(&wfull[s], (((iw - 1 - s) / C::kSW)) & 1, 705);
    }
  } else if (warp == kXWarp) {
    // ------------------------------- activation producer (TMA) -------------------------------
    // One [kMP tokens x 128] bf16 tile per unit (two 64-column 128B-swizzled boxes; rows >= m and columns
    // >= K read as zero), into a ring of kSX stages once the phase's input is final. A thread of its own,
    // so the weight stream never waits for an activation phase and vice versa. TMA writes through the async
    // proxy, like the MMA reads: the ring's mbarriers order the two, no proxy fence is needed here.
    if (lane == 0) {
      griddep_wait();
      trace(1);
      int ready_ph = -1;  // phases are taken in order: every phase <= ready_ph is known ready
      int ix = 0;
      for (Cur kx = cur_begin(p, c); kx.ph < kNLin && !s_abort; cur_advance(p, c, kx), ++ix) {
        const int s = ix % C::kSX;
        if (ix >= C::kSX && !mbar_wait_ab(cx, &xempty[s], ((ix / C::kSX) - 1) & 1, 706, (uint32_t)ix)) break;
        if (kx.ph > ready_ph) {
          uint64_t t0 = 0;
          bool rdy = false;
          for (uint32_t spin = 0; !(rdy = x_ready(p, kx.ph, kx.u)); ++spin) {
            if ((spin & 7) == 7) {
              if (s_abort || *reinterpret_cast<volatile int*>(&g_mg_dev_error) != 0) break;
              const uint64_t t = global_ns();
              if (!t0) t0 = t;
              else if (t - t0 > p.timeout_ns) {
                fail(cx, 701, (uint32_t)ix, ((uint32_t)(kx.ph & 0xff) << 24) | (uint32_t)kx.u);
                break;
              }
              __nanosleep(64);
            }
          }
          if (!rdy) {
            s_abort = 1;
            break;
          }
          // the phase's input was written through the generic proxy (and fenced by its writers): order this
          // thread's TMA reads after the acquire that saw it complete
          fence_proxy_async_global();
          ready_ph = kx.ph;
          trace(2 + kx.ph);  // 2 O, 3 gate/up, 4 down, 5 QKV: first activation tile requested
        }
        uint8_t* sx = smem + C::kXOff + s * C::kXBytes;
        const int k0 = kx.kb * kBK;
        mbar_arrive_expect_tx(&xfull[s], C::kXBytes);
        tma_load_2d(sx, &maps.x[kx.ph], &xfull[s], k0, 0);
        tma_load_2d(sx + kMP * 128, &maps.x[kx.ph], &xfull[s], k0 + 64, 0);
        if ((ix & 7) == 7) prog(0, (uint32_t)(ix + 1));
      }
      // shared memory is the destination of every load issued: all of them land before the CTA exits
      for (int s = 0; s < C::kSX && s < ix; ++s) mbar_wait(&xfull[s], (((ix - 1 - s) / C::kSX)) & 1, 707);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      int i = 0, seg = 0;
      for (Cur k = cur_begin(p, c); k.ph < kNLin && !s_abort; cur_advance(p, c, k), ++i) {
        const bool first = k.u == k.u0 || k.kb == 0;
        const bool last = k.u + 1 == k.u1 || k.kb + 1 == k.KB;
        const int buf = seg & 1;
        const uint32_t where_u = ((uint32_t)(k.ph & 0xff) << 24) | (uint32_t)k.u;
        if (first && seg >= 2 && !mbar_wait_ab(cx, &accempty[buf], ((seg >> 1) - 1) & 1, 710, i, where_u)) break;
        if (!mbar_wait_ab(cx, &xfull[i % C::kSX], (i / C::kSX) & 1, 711, i, where_u)) break;
        if (!mbar_wait_ab(cx, &afull[i % C::kNA], (i / C::kNA) & 1, 712, i, where_u)) break;
        tc_fence_after();
        const uint32_t sx = smem_u32(smem + C::kXOff + (i % C::kSX) * C::kXBytes);
        const uint32_t ab = (uint32_t)(i % C::kNA);
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j) {
          const uint32_t a_t = tmem + ab * 64 + (uint32_t)(j * 8);
          const uint64_t bd = desc_sw128(sx + (uint32_t)((j >> 2) * kMP * 128 + (j & 3) * 32));
          tc_mma_ts(tmem + C::kAcc0 + (uint32_t)(buf * kMP), a_t, bd, C::kIdesc, (first && j == 0) ? 0u : 1u);
        }
        tc_commit(&xempty[i % C::kSX]);
        tc_commit(&aempty[i % C::kNA]);
        if (last) {
          tc_commit(&accfull[buf]);
          ++seg;
          prog(2, (uint32_t)(i + 1) | ((uint32_t)seg << 16));
        }
      }
      trace(6);  // MMA issue done
      if (i > 0) {  // TMEM is freed at exit: no MMA may still be writing it
        tc_commit(mma_fin);
        mbar_wait(mma_fin, 0, 715);
      }
    }
  } else if (warp < kConvWarps) {
    // ------------------------------- converters -------------------------------
    const int row = (warp & 3) * 32 + lane;
    const int hh = warp >> 2;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    int i = 0;
    for (Cur k = cur_begin(p, c); k.ph < kNLin; cur_advance(p, c, k), ++i) {
      const int s = i % C::kSW, ab = i % C::kNA;
      // wait results are made warp-uniform: the tcgen05 stores below need the whole warp
      if (!__all_sync(0xffffffffu, mbar_wait_ab(cx, &wfull[s], (i / C::kSW) & 1, 720))) break;
      const uint8_t* src = smem + s * kWBytes + row * 128;
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
      // The stage is released only after its bytes have been consumed (converted): an arrive right after the
      // shared loads were issued could let the producer's next TMA write land before a load returned.
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[s]);
      if (i >= C::kNA && !__all_sync(0xffffffffu, mbar_wait_ab(cx, &aempty[ab], ((i / C::kNA) - 1) & 1, 721)))
        break;
      tmem_st32(tmem + lane_base + (uint32_t)(ab * 64 + hh * 32), r);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ab]);
      if (warp == 0 && lane == 0 && (i & 7) == 7) prog(1, (uint32_t)(i + 1));
    }
    if (warp == 0 && lane == 0) trace(14);  // conversion done
  } else {
    // ------------------------------- epilogue warps -------------------------------
    const int e = epi_row();  // weight row within the tile == this thread's TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    griddep_wait();
    // all-reduce epochs of this launch's row-parallel linears (world > 1): O then down
    uint32_t ep_o = 0, ep_dn = 0;
    if (p.po.world > 1) {
      const uint32_t cnt = *reinterpret_cast<volatile uint32_t*>(p.po.count);
      ep_o = (p.flags & MG_BLK_O) ? cnt + 1u : 0u;
      ep_dn = (p.flags & MG_BLK_MLP) ? cnt + 1u + (ep_o ? 1u : 0u) : 0u;
    }
    int seg = 0;
    bool ok = true;  // uniform over the 128 epilogue threads
    // This CTA's segments of linear `ph`; returns false (for all threads) once the CTA aborted.
    auto run_segments = [&](int ph, uint32_t epoch) -> bool {
      const Lin& L = p.lin[ph];
      const int64_t u0 = rstart(L.units, c, p.G), u1 = rstart(L.units, c + 1, p.G);
      for (int64_t u = u0; u < u1;) {
        const int t = (int)(u / L.kb);
        const int64_t u_end = std::min<int64_t>(u1, (int64_t)(t + 1) * L.kb);
        const uint32_t nk = (uint32_t)(u_end - u);
        const int buf = seg & 1;
        if (e == 0) prog(3, (uint32_t)seg | ((uint32_t)(ph == L_O ? 0 : ph == L_GU ? 2 : ph == L_DN ? 3 : 5) << 16) |
                            (1u << 31));
        const bool got = __all_sync(0xffffffffu, mbar_wait_ab(cx, &accfull[buf], (seg >> 1) & 1, 730, seg,
                                                              ((uint32_t)ph << 24) | (uint32_t)u));
        ++seg;
        if (got) {
          tc_fence_after();
          uint32_t r[kMP];
          tmem_ld32(tmem + lane_base + C::kAcc0 + (uint32_t)(buf * kMP), r);
          tc_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[buf]);
          // park the partial, count the K blocks in; the CTA completing the ticket finishes the tile
          const int slot = c - owner(L.units, (int64_t)t * L.kb, p.G);
          float4* dst = reinterpret_cast<float4*>(L.part + (((int64_t)t * L.maxslots + slot) * kBN + e) * kMP);
#pragma unroll
          for (int q = 0; q < kMP / 4; ++q)
            dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                 __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
          __threadfence();
        }
        epi_bar();
        if (e == 0) {
          s_stop = s_abort;
          s_flag = !s_stop && atom_add_acq_rel(L.ticket + t, nk) + nk == (uint32_t)L.kb;
        }
        epi_bar();
        if (*reinterpret_cast<volatile int*>(&s_stop)) return false;
        if (*reinterpret_cast<volatile int*>(&s_flag)) {
          __threadfence();
          finish_tile(p, cx, ph, t, stg, epoch);
        }
        u = u_end;
        if (e == 0) prog(3, (uint32_t)seg | ((uint32_t)(ph == L_O ? 0 : ph == L_GU ? 2 : ph == L_DN ? 3 : 5) << 16));
      }
      return true;
    };
    // Token row c's norm, once `target` tiles of the feeding linear are final (counter `done`).
    auto norm_phase = [&](const uint32_t* done, uint32_t target, int where, const float* w, const float* wb,
                          const float* rp_bias, uint32_t epoch, __nv_bfloat16* x, uint32_t* out_count) -> bool {
      if (e == 0) prog(3, (uint32_t)seg | ((where == 740 ? 1u : 4u) << 16) | (1u << 31));
      if (e == 0 && done) wait_ge(cx, done, target, where);
      bool go = !epi_stop(&s_abort, &s_stop);
      __threadfence();
      if (go) go = norm_row(p, cx, c, w, wb, rp_bias, epoch, x, s_red, &s_stop);
      fence_proxy_async_global();
      __threadfence();
      epi_bar();
      if (e == 0) atom_add_acq_rel(out_count, 1u);
      return go;
    };
    if (e == 0) trace(7);
    if (p.flags & MG_BLK_O) ok = run_segments(L_O, ep_o);
    if (e == 0) trace(8);  // O drained
    if (ok && (p.flags & MG_BLK_MLP)) {
      if (c < p.m)
        ok = norm_phase((p.flags & MG_BLK_O) ? p.ctl + C_O_DONE : nullptr, (uint32_t)p.lin[L_O].tiles, 740,
                        p.n2_w, p.n2_b, p.lin[L_O].bias, ep_o, p.x2, p.ctl + C_N2_DONE);
      if (e == 0) trace(9);  // N2 done (or skipped)
      if (ok) ok = run_segments(L_GU, 0);
      if (e == 0) trace(10);  // gate/up drained
      if (ok) ok = run_segments(L_DN, ep_dn);
      if (e == 0) trace(11);  // down drained
    }
    if (ok && (p.flags & MG_BLK_N1) && c < p.m)
      ok = norm_phase((p.flags & MG_BLK_MLP) ? p.ctl + C_DN_DONE : nullptr, (uint32_t)p.lin[L_DN].tiles, 741,
                      p.n1_w, p.n1_b, p.lin[L_DN].bias, ep_dn, p.x1, p.ctl + C_N1_DONE);
    if (e == 0) trace(12);  // N1 done (or skipped)
    if (ok && (p.flags & MG_BLK_QKV)) ok = run_segments(L_QKV, 0);
    if (e == 0) trace(13);  // QKV drained
    if (e == 0) prog(3, (uint32_t)seg | (6u << 16));
  }

  // ------------------------------- exit -------------------------------
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    s_flag = atom_add_acq_rel(p.ctl + C_EXIT, 1u) == (uint32_t)(p.G - 1);
    // the last CTA out advances the all-reduce count past this launch's epochs
    if (s_flag && p.po.world > 1) {
      const uint32_t n_ar = ((p.flags & MG_BLK_O) ? 1u : 0u) + ((p.flags & MG_BLK_MLP) ? 1u : 0u);
      *reinterpret_cast<volatile uint32_t*>(p.po.count) += n_ar;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) trace(15);
  if (s_flag) {  // every other CTA is past its last use of the control words: leave them at zero
    for (int i = threadIdx.x; i < p.ctl_words; i += kThreads) p.ctl[i] = 0u;
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
int sm_count_blk() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

struct Plan {
  Lin lin[kNLin];
  size_t ctl_words, ws_bytes, part_off[kNLin];
  int G;
};

int64_t ceil128(int64_t v) { return (v + 127) / 128; }

constexpr size_t kCtlBytes = 64 * 1024;  // control words of every plan (16384 tiles and flags at most)

int max_slots(int64_t units, int kb, int G) {
  int mx = 1;
  const int64_t tiles = units / kb;
  for (int64_t t = 0; t < tiles; ++t) {
    const int64_t a = t * kb, b = a + kb - 1;
    const int ca = (int)(((a + 1) * G - 1) / units), cb = (int)(((b + 1) * G - 1) / units);
    mx = std::max(mx, cb - ca + 1);
  }
  return mx;
}

int on_host(const mg_block_args* a, int ph) {
  switch (ph) {
    case L_O: return a->flags & MG_BLK_O;
    case L_GU:
    case L_DN: return a->flags & MG_BLK_MLP;
    default: return a->flags & MG_BLK_QKV;
  }
}

const mg_block_linear& lin_arg(const mg_block_args* a, int ph) {
  switch (ph) {
    case L_O: return a->o;
    case L_GU: return a->gate_up;
    case L_DN: return a->down;
    default: return a->qkv;
  }
}

int check_and_plan(const mg_block_args* a, Plan* pl) {
  if (!a) return MG_ERR_INVALID_ARG;
  const int flags = a->flags;
  if (flags & ~(MG_BLK_O | MG_BLK_MLP | MG_BLK_N1 | MG_BLK_QKV) || !flags) return MG_ERR_INVALID_ARG;
  if (a->m < 0 || a->m > kMP) return a->m < 0 ? MG_ERR_INVALID_ARG : MG_ERR_UNSUPPORTED;
  if (a->m > sm_count_blk()) return MG_ERR_UNSUPPORTED;  // one norm row per CTA
  const int H = a->hidden;
  if (H <= 0 || H % 128 || !a->h) return MG_ERR_INVALID_ARG;
  if (a->norm != MG_NORM_RMS && a->norm != MG_NORM_LAYER) return MG_ERR_INVALID_ARG;
  const int D = a->head_dim;
  if ((flags & (MG_BLK_O | MG_BLK_QKV)) && (a->hq <= 0 || a->hkv <= 0 || a->hq % a->hkv || (D != 32 && D != 64 && D != 128)))
    return MG_ERR_INVALID_ARG;
  const int G = sm_count_blk();
  if (G > 256) return MG_ERR_UNSUPPORTED;  // unit arithmetic on the device is 32-bit: units * G < 2^32
  pl->G = G;
  size_t words = C_HDR;
  for (int ph = 0; ph < kNLin; ++ph) {
    Lin& L = pl->lin[ph];
    L = Lin{};
    if (!on_host(a, ph)) continue;
    const mg_block_linear& s = lin_arg(a, ph);
    if (!s.packed || !s.scales || s.n <= 0 || s.k <= 0 || s.k % 16) return MG_ERR_INVALID_ARG;
    if (ph != L_QKV && s.n % 128) return MG_ERR_INVALID_ARG;  // only QKV may end in a partial tile
    if (reinterpret_cast<uintptr_t>(s.packed) & 15) return MG_ERR_INVALID_ARG;
    L.scales = s.scales;
    L.bias = s.bias;
    L.tiles = (int)ceil128(s.n);
    L.kb = (int)ceil128(s.k);
    L.units = (int64_t)L.tiles * L.kb;
    if (L.units * kBN > 0x7fffffffLL) return MG_ERR_UNSUPPORTED;
    L.maxslots = max_slots(L.units, L.kb, G);
    words += (size_t)L.tiles;  // tickets
  }
  // shapes tying the phases together
  if (flags & MG_BLK_O) {
    if (a->o.k != (int64_t)a->hq * D || a->o.n != H || !a->attn) return MG_ERR_INVALID_ARG;
  }
  if (flags & MG_BLK_MLP) {
    const bool swi = a->mlp == MG_EPI_SWIGLU_BF16;
    if (!swi && a->mlp != MG_EPI_GELU_BF16) return MG_ERR_INVALID_ARG;
    if (a->gate_up.k != H || a->down.n != H || !a->x2 || !a->act || !a->n2_w) return MG_ERR_INVALID_ARG;
    if (a->down.k != (swi ? a->gate_up.n / 2 : a->gate_up.n)) return MG_ERR_INVALID_ARG;
    if (a->norm == MG_NORM_LAYER && !a->n2_b) return MG_ERR_INVALID_ARG;
  }
  if (flags & MG_BLK_N1) {
    if (!a->n1_w || !a->x1 || (a->norm == MG_NORM_LAYER && !a->n1_b)) return MG_ERR_INVALID_ARG;
  }
  if (flags & MG_BLK_QKV) {
    const int64_t nqkv = (int64_t)(a->hq + 2 * a->hkv) * D;
    if (a->qkv.k != H || nqkv != a->qkv.n || !a->x1 || !a->q_out || !a->k_pool || !a->v_pool ||
        !a->slots || a->num_blocks <= 0)
      return MG_ERR_INVALID_ARG;
    if (a->cos_sin && (!a->positions || a->max_pos <= 0)) return MG_ERR_INVALID_ARG;
  }
  // workspace: a fixed control region (tickets, flags, counters), then the partial slots of each linear.
  // The region's size does not depend on the plan: launches of different plans share one workspace, and
  // no launch may leave partials where another launch's control words live.
  if (words * 4 > kCtlBytes) return MG_ERR_UNSUPPORTED;
  size_t off = kCtlBytes;
  pl->ctl_words = words;
  for (int ph = 0; ph < kNLin; ++ph) {
    pl->part_off[ph] = off;
    if (pl->lin[ph].tiles) off += (size_t)pl->lin[ph].tiles * pl->lin[ph].maxslots * kMP * kBN * 4;
  }
  pl->ws_bytes = off;
  return MG_OK;
}

}  // namespace

extern "C" int mg_decode_block_workspace_bytes(const mg_block_args* a, size_t* bytes) {
  if (!bytes) return MG_ERR_INVALID_ARG;
  Plan pl;
  const int rc = check_and_plan(a, &pl);
  if (rc) return rc;
  *bytes = pl.ws_bytes;
  return MG_OK;
}

extern "C" int mg_decode_block(const mg_block_args* a, void* comm, void* workspace, size_t workspace_bytes,
                               void* stream) {
  Plan pl;
  int rc = check_and_plan(a, &pl);
  if (rc) return rc;
  if (!workspace || workspace_bytes < pl.ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return MG_ERR_INVALID_ARG;
  if (a->m == 0) return MG_OK;
  Params p{};
  if (comm) {
    rc = mg_comm_peer_out(comm, &p.po);
    if (rc) return rc;
    if ((int64_t)a->m * a->hidden > 2 * p.po.slot) return MG_ERR_INVALID_ARG;
  } else {
    p.po.world = 1;
  }
  static bool attr_done[64] = {};
  static std::mutex attr_mu;
  MG_CUDA_TRY(mg_once_per_device(attr_done, attr_mu, [] {
    return cudaFuncSetAttribute(decode_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BlkCfg::kSmem);
  }));
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  const void* xsrc[kNLin] = {a->attn, a->x2, a->act, a->x1};
  char* ws = static_cast<char*>(workspace);
  uint32_t* ctl = reinterpret_cast<uint32_t*>(ws);
  size_t word = C_HDR;
  for (int ph = 0; ph < kNLin; ++ph) {
    Lin& L = pl.lin[ph];
    if (!L.tiles) continue;
    const mg_block_linear& s = lin_arg(a, ph);
    L.part = reinterpret_cast<float*>(ws + pl.part_off[ph]);
    L.ticket = ctl + word;
    word += L.tiles;
    rc = mg_make_map_2d(&maps.w[ph], CU_TENSOR_MAP_DATA_TYPE_UINT8, s.packed, kBK, (uint64_t)(L.units * kBN), kBK,
                        kBK, kBN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (!xsrc[ph] || (reinterpret_cast<uintptr_t>(xsrc[ph]) & 15)) return MG_ERR_INVALID_ARG;
    rc = mg_make_map_2d(&maps.x[ph], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xsrc[ph], (uint64_t)s.k, (uint64_t)a->m,
                        (uint64_t)s.k * 2, 64, kMP, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    L.k = (int)s.k;
  }
  p.m = a->m;
  p.flags = a->flags;
  p.hidden = a->hidden;
  p.act_cols = (a->flags & MG_BLK_MLP) ? (int)a->down.k : 0;
  p.nqkv = (a->hq + 2 * a->hkv) * a->head_dim;
  p.hq = a->hq;
  p.hkv = a->hkv;
  p.d = a->head_dim;
  p.norm = a->norm;
  p.mlp = a->mlp;
  p.G = pl.G;
  p.ctl_words = (int)pl.ctl_words;
  p.max_pos = a->max_pos;
  p.eps = a->eps;
  for (int ph = 0; ph < kNLin; ++ph) p.lin[ph] = pl.lin[ph];
  p.h = a->h;
  p.n2_w = a->n2_w;
  p.n2_b = a->n2_b;
  p.n1_w = a->n1_w;
  p.n1_b = a->n1_b;
  p.x2 = static_cast<__nv_bfloat16*>(a->x2);
  p.x1 = static_cast<__nv_bfloat16*>(a->x1);
  p.act = static_cast<__nv_bfloat16*>(a->act);
  p.cos_sin = a->cos_sin;
  p.positions = a->positions;
  p.slots = a->slots;
  p.q_out = a->q_out;
  p.k_pool = static_cast<__nv_bfloat16*>(a->k_pool);
  p.v_pool = static_cast<__nv_bfloat16*>(a->v_pool);
  p.num_blocks = a->num_blocks;
  p.ctl = ctl;
  // a wait inside the CTA may sit behind a peer wait (bounded by the communicator's limit) on another CTA
  p.timeout_ns = 2000000000ull + (p.po.world > 1 ? 2 * p.po.timeout_ns : 0ull);
  MG_CUDA_TRY(mg_launch(decode_block_kernel, dim3((unsigned)pl.G), dim3(kThreads), BlkCfg::kSmem, mg_stream(stream), 1,
                        maps, p));
  return MG_OK;
}

extern "C" int mg_decode_block_diag(uint32_t* out, int clear) {
  if (!out) return MG_ERR_INVALID_ARG;
  MG_CUDA_TRY(cudaMemcpyFromSymbol(out, g_blk_diag, sizeof(uint32_t) * 32));
  MG_CUDA_TRY(cudaMemcpyFromSymbol(out + 32, g_blk_snap, sizeof(uint32_t) * kDiagCtas * 4));
  if (clear) {
    static const uint32_t zeros[32] = {};
    MG_CUDA_TRY(cudaMemcpyToSymbol(g_blk_diag, zeros, sizeof(zeros)));
  }
  return MG_OK;
}

extern "C" int mg_decode_block_trace(uint64_t* out, int ctas) {
  if (!out || ctas <= 0 || ctas > kDiagCtas) return MG_ERR_INVALID_ARG;
  MG_CUDA_TRY(cudaMemcpyFromSymbol(out, g_blk_ts, sizeof(uint64_t) * kTracePoints * ctas));
  return MG_OK;
}
