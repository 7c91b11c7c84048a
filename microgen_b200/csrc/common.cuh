// Shared device helpers for the sm_100a kernels of libmicrogen_b200.
//
// Every wait a kernel spins on (mbarrier phases, peer flags) is bounded: after
// MG_SPIN_LIMIT polls it records MG_ERR_TIMEOUT in the device error word and
// the caller unwinds, so a wait that can never complete ends in an error
// status the host reads instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

#include "../../include/microgen_b200.h"

#define MG_SPIN_LIMIT (1u << 22)

// Device-side error word (first error wins). Read by mg_device_error().
extern __device__ int g_mg_dev_error;
extern __device__ int g_mg_dev_error_info;

__device__ __forceinline__ void mg_record_error(int code, int info) {
  if (atomicCAS(&g_mg_dev_error, 0, code) == 0) g_mg_dev_error_info = info;
}

// Host-side: remember the last CUDA error for mg_last_cuda_error().
int mg_set_cuda_error(cudaError_t e);
#define MG_CUDA_TRY(expr)                                  \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return mg_set_cuda_error(_e);   \
  } while (0)
#define MG_LAUNCH_CHECK() MG_CUDA_TRY(cudaGetLastError())

static inline cudaStream_t mg_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch. Every kernel of the decode step is launched with programmatic
// stream serialization: it may start while its predecessor drains, signals its own dependents at
// entry (griddep_launch), and calls griddep_wait before it touches anything a predecessor
// writes. Every kernel waits (even on early-exit paths), so the completion of a kernel implies
// the completion of the whole chain before it. MG_PDL=0 in the environment turns it off.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool mg_pdl_enabled();

// Runs `setup` (returning a cudaError_t) once per device for one `flags` array: function attributes
// such as the dynamic shared-memory limit belong to the current device's copy of a kernel. Threads
// that get here first on a device wait for the set-up under a lock; the device is only marked done
// after `setup` succeeded, so a failed set-up is retried by the next call.
template <typename F>
inline cudaError_t mg_once_per_device(bool (&flags)[64], std::mutex& mu, F&& setup) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return setup();
  std::lock_guard<std::mutex> lock(mu);
  if (flags[dev]) return cudaSuccess;
  e = setup();
  if (e == cudaSuccess) flags[dev] = true;
  return e;
}

// Host: a 2-D tiled TMA descriptor (row-major [outer][inner], row_bytes apart; box_inner x box_outer).
int mg_make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

template <typename... KArgs, typename... Args>
static inline cudaError_t mg_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                    unsigned cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  unsigned n = 0;
  if (cluster > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  if (mg_pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------------------------
// Peer-memory exchange of the row-parallel linears (tensor parallelism over NVLink / NVSwitch).
// Every rank owns one device allocation, mapped into every other rank's process through CUDA IPC:
//   recv  u64 [2 sets][world][slot]   rank r's partial of all-reduce e lands in set e%2, slot r
// plus two local counters (all-reduces pushed by this rank; CTAs done in the push under way).
// Each receive word carries its own flag: low half = two adjacent partial values as bf16 (the
// precision the reference's all-reduce of bf16 linear outputs has), high half = the epoch e of the
// all-reduce that wrote it. An aligned 64-bit store is single-copy atomic, so a reader that sees
// epoch e in a word also sees that word's values; no fence or separate flag is needed.
// ---------------------------------------------------------------------------------------------
#define MG_MAX_RANKS 8
#define MG_EPI_PEER_F32 5  // internal epilogue: push acc*scale to every rank's receive slot

struct PeerOut {
  uint64_t* recv[MG_MAX_RANKS];    // each rank's receive area, as mapped in this process
  uint32_t* count;                 // this rank: all-reduces pushed so far (= epoch of the last one)
  uint32_t* done;                  // this rank: CTAs finished in the push under way
  int64_t slot;                    // words (value pairs) per (set, rank) slot
  uint64_t timeout_ns;             // how long a reduce waits for a peer's words before giving up
  int rank, world;
};

// Host: the PeerOut of a communicator made by mg_comm_create / mg_comm_open (comm.cu).
int mg_comm_peer_out(void* comm, PeerOut* out);

__device__ __forceinline__ void st_volatile_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_volatile_v2u64(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_volatile_v2u64(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------
// Small math helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// torch.argmax's order of (value, index) candidates: NaN above every number, equal values (or two
// NaNs) by the smaller index. True when (v, i) comes before (best, bi).
__device__ __forceinline__ bool mg_argmax_better(float v, int32_t i, float best, int32_t bi) {
  const bool vn = v != v, bn = best != best;
  if (vn != bn) return vn;
  return (!vn && v > best) || ((vn || v == best) && i < bi);
}

// bf16x2 word -> two floats (exact: bf16 is the upper half of an fp32)
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Two floats -> bf16x2 (round to nearest even), lo in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Four signed int8 packed in a word -> four exact floats via the 2^23 magic:
// (0x4B000000 | (b ^ 0x80)) is 2^23 + b + 128 exactly; subtracting 2^23 + 128 leaves b.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t u = w ^ 0x80808080u;
  const float magic = 8388736.0f;  // 2^23 + 128
  f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - magic;
  f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - magic;
  f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - magic;
  f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - magic;
}

// Four signed int8 -> two bf16x2 words (exact: |b| <= 128 fits bf16's 8-bit significand).
// The fp32 values are small integers, so truncating to the upper 16 bits is exact.
// 8 instructions per 4 bytes: byte b is placed in a bf16 with bits 0x43 : (b & 0x7F), i.e. the value
// 128 + (b & 0x7F); subtracting 128 (b >= 0) or 256 (b < 0) — a second bf16 whose bit 7 is b's sign
// bit — leaves b. Every operand and the difference are small integers, so the bf16 subtraction is exact.
__device__ __forceinline__ uint32_t i8x2_to_bf16x2(uint32_t p) {  // p: halves hold bytes (0x00bb)
  const uint32_t v = (p & 0x007F007Fu) | 0x43004300u;
  const uint32_t m = (p & 0x00800080u) | 0x43004300u;
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(m));
  return r;
}
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = i8x2_to_bf16x2(__byte_perm(w, 0u, 0x4140));  // b0 (low half), b1
  hi = i8x2_to_bf16x2(__byte_perm(w, 0u, 0x4342));  // b2, b3
}

// ---------------------------------------------------------------------------------------------
// Shared-memory / mbarrier PTX wrappers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking probe of a phase (no suspension), for threads that poll several barriers.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait. Returns false (and records MG_ERR_TIMEOUT with `where`) if the phase never flips.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int where) {
  for (uint32_t i = 0; i < MG_SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  mg_record_error(MG_ERR_TIMEOUT, where);
  return false;
}

// ---------------------------------------------------------------------------------------------
// TMA (tiled tensor copies, no multicast)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// Untiled bulk copy global -> this CTA's shared memory (no multicast): both addresses 16-byte aligned,
// bytes a multiple of 16; completes `bytes` of the barrier's transaction count.
__device__ __forceinline__ void bulk_load_smem(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* holder_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]ᵀ, kind::f16 (bf16 inputs, fp32 accumulate), one CTA.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]ᵀ
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier of this CTA once every previously issued tcgen05.mma of this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp <-> lane (warp base + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// Thread-block cluster helpers (distributed shared memory)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Distributed-shared-memory loads. `volatile` keeps them on their side of the cluster barriers
// (themselves volatile asm); no memory clobber, so independent loads can be issued back to back.
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
