// Peer-memory communicator and the reduce(+norm) half of the fused row-parallel all-reduce.
//
// The push half lives in the tcgen05 linear's MG_EPI_PEER_F32 epilogue (i8_linear.cu): every CTA
// stores its output tile (scale applied, no bias) into slot [e%2][my rank] of every rank's receive
// area over NVLink as 64-bit words {two bf16 values, epoch e}; the last CTA of the launch advances
// this rank's count to e.
//
// rowpar_reduce_norm_kernel reads e from the count, waits (bounded by time) until each word it
// needs carries epoch e, sums the world partials in rank order onto the fp32 residual (identical
// bits on every rank), adds the bias once, and applies the next RMSNorm / LayerNorm, writing bf16
// activations for the next linear. No fences and no separate flags are involved: each word is its
// own flag.
//
// Reuse of a set is safe without extra handshakes: a rank pushes e+2 only after its reduce e+1 saw
// every peer's words of e+1, and a peer pushes e+1 only after its own reduce e consumed set e%2.
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace {

constexpr int kThreads = 1024;              // most: one float4 of a row per thread at hidden <= 4096
constexpr int kMaxV = 2;                     // float4 per thread: rows up to 8192
// A peer that has not pushed within the communicator's limit is reported: MG_PEER_TIMEOUT_MS in the
// environment of mg_comm_create (default 1000 ms; ranks whose host sides drift apart by more than that,
// e.g. through uneven start-up work, need a larger value).
constexpr uint64_t kDefaultWaitNs = 1000000000ull;

struct Comm {
  int rank = 0, world = 1, device = 0;
  int64_t slot = 0;
  uint64_t timeout_ns = kDefaultWaitNs;
  size_t recv_bytes = 0, bytes = 0;
  char* base = nullptr;
  cudaIpcMemHandle_t handle{};
  char* peer[MG_MAX_RANKS] = {};
  bool opened[MG_MAX_RANKS] = {};
  bool ready = false;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
  if (w == 0) r = warp_sum(r);
  if (threadIdx.x == 0) red[0] = r;
  __syncthreads();
  return red[0];
}

// Waits until the two words at p (four values, 16-byte aligned) carry `epoch`. Gives up once `dead`
// is set or the wait has run for limit_ns, recording MG_ERR_TIMEOUT with the peer rank in the detail.
__device__ __forceinline__ void wait_words(const uint64_t* p, uint32_t epoch, uint64_t (&wd)[2], uint64_t& t0,
                                           bool& dead, int r, uint64_t limit_ns) {
  for (uint32_t spin = 0;; ++spin) {
    ld_volatile_v2u64(p, wd[0], wd[1]);
    if (dead || ((uint32_t)(wd[0] >> 32) == epoch && (uint32_t)(wd[1] >> 32) == epoch)) return;
    if ((spin & 31) == 31) {
      const uint64_t t = global_ns();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > limit_ns) {
        mg_record_error(MG_ERR_TIMEOUT, 600 + r);
        dead = true;
        return;
      }
      __nanosleep(64);
    }
  }
}

// One CTA per token row (blockDim: the row's float4 count rounded up to a warp, at most kThreads).
// Each thread loads its words from every rank before it consumes any, so the world's words cost one
// memory round trip rather than one per rank. norm: 0 = none, 1 = RMSNorm (w), 2 = LayerNorm (w, wb).
__global__ void __launch_bounds__(kThreads) rowpar_reduce_norm_kernel(PeerOut po, float* __restrict__ h,
                                                                       const float* __restrict__ bias, int n,
                                                                       int norm, const float* __restrict__ w,
                                                                       const float* __restrict__ wb, float eps,
                                                                       __nv_bfloat16* __restrict__ x) {
  __shared__ float red[32];
  griddep_launch();
  griddep_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(po.count);
  const int64_t row = blockIdx.x;
  const uint64_t* recv = po.recv[po.rank] + (int64_t)(epoch & 1u) * po.world * po.slot + row * (n / 2);
  float* hr = h + row * n;
  const int nv = n >> 2;
  uint64_t t0 = 0;
  bool dead = false;
  float4 v[kMaxV];
  float s1 = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxV; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < nv) {
      float4 a = reinterpret_cast<const float4*>(hr)[idx];
      uint64_t wd[MG_MAX_RANKS][2];
#pragma unroll
      for (int r = 0; r < MG_MAX_RANKS; ++r)  // every rank's words in flight at once
        if (r < po.world) ld_volatile_v2u64(recv + (int64_t)r * po.slot + idx * 2, wd[r][0], wd[r][1]);
#pragma unroll
      for (int r = 0; r < MG_MAX_RANKS; ++r) {
        if (r >= po.world) break;
        if ((uint32_t)(wd[r][0] >> 32) != epoch || (uint32_t)(wd[r][1] >> 32) != epoch)
          wait_words(recv + (int64_t)r * po.slot + idx * 2, epoch, wd[r], t0, dead, r, po.timeout_ns);
        a.x += bf16lo((uint32_t)wd[r][0]);
        a.y += bf16hi((uint32_t)wd[r][0]);
        a.z += bf16lo((uint32_t)wd[r][1]);
        a.w += bf16hi((uint32_t)wd[r][1]);
      }
      if (bias) {
        const float4 b = reinterpret_cast<const float4*>(bias)[idx];
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      reinterpret_cast<float4*>(hr)[idx] = a;
      v[i] = a;
      s1 += norm == 2 ? (a.x + a.y + a.z + a.w) : (a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w);
    }
  }
  if (norm == 0) return;
  float mean = 0.f, inv;
  if (norm == 1) {
    inv = rsqrtf(block_sum(s1, red) / (float)n + eps);
  } else {
    mean = block_sum(s1, red) / (float)n;
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxV; ++i) {
      const int idx = threadIdx.x + i * blockDim.x;
      if (idx < nv) {
        const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
        s2 += a * a + b * b + c * c + d * d;
      }
    }
    inv = rsqrtf(block_sum(s2, red) / (float)n + eps);
  }
  __nv_bfloat16* xr = x + row * n;
#pragma unroll
  for (int i = 0; i < kMaxV; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < nv) {
      const float4 g = reinterpret_cast<const float4*>(w)[idx];
      float4 o;
      if (norm == 1) {
        o = make_float4(g.x * (v[i].x * inv), g.y * (v[i].y * inv), g.z * (v[i].z * inv), g.w * (v[i].w * inv));
      } else {
        const float4 b = reinterpret_cast<const float4*>(wb)[idx];
        o = make_float4((v[i].x - mean) * inv * g.x + b.x, (v[i].y - mean) * inv * g.y + b.y,
                        (v[i].z - mean) * inv * g.z + b.z, (v[i].w - mean) * inv * g.w + b.w);
      }
      uint2 u;
      u.x = pack_bf16x2(o.x, o.y);
      u.y = pack_bf16x2(o.z, o.w);
      reinterpret_cast<uint2*>(xr)[idx] = u;
    }
  }
}

// Greedy argmax over a vocab-parallel lm_head: rank r holds logits columns [offset_r, offset_r + n_r) of
// every row, in rank order. idx[i] enters as this rank's first maximal column of row i (mg_argmax_rows over
// the shard). Each row's {value, global index} goes to slot [e%2][my rank] of every rank's receive area as two
// words tagged with epoch e (e = this rank's count + 1, the same sequence the row-parallel pushes use); then
// each row waits for the world's records (bounded by time), keeps the largest value (NaN above every
// number), the smallest global index on ties (torch.argmax's first maximal index over the whole row,
// pytorch.py:153-155), and the count advances to e. One CTA, one thread per row.
__global__ void __launch_bounds__(1024) vocab_argmax_merge_kernel(PeerOut po, const float* __restrict__ logits,
                                                                   int64_t ld, int64_t n_local, int64_t offset,
                                                                   int32_t* __restrict__ idx, int m) {
  griddep_launch();
  griddep_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(po.count) + 1u;
  const uint64_t tag = (uint64_t)epoch << 32;
  const int i = threadIdx.x;
  if (i < m) {
    int32_t li = idx[i];
    float v = -INFINITY;
    if (li >= 0 && li < n_local) {
      v = logits[(int64_t)i * ld + li];
    } else {
      mg_record_error(MG_ERR_DEVICE, 660);
      li = 0;
    }
    const int64_t off = ((int64_t)(epoch & 1u) * po.world + po.rank) * po.slot + 2 * (int64_t)i;
    const uint64_t w0 = tag | __float_as_uint(v), w1 = tag | (uint32_t)(li + offset);
    for (int r = 0; r < po.world; ++r) st_volatile_v2u64(po.recv[r] + off, w0, w1);
    const uint64_t* recv = po.recv[po.rank] + (int64_t)(epoch & 1u) * po.world * po.slot + 2 * (int64_t)i;
    float best = -INFINITY;
    int32_t bi = 0x7fffffff;
    uint64_t t0 = 0;
    bool dead = false;
    uint64_t wd[MG_MAX_RANKS][2];
#pragma unroll
    for (int r = 0; r < MG_MAX_RANKS; ++r)  // every rank's record in flight at once
      if (r < po.world) ld_volatile_v2u64(recv + (int64_t)r * po.slot, wd[r][0], wd[r][1]);
#pragma unroll
    for (int r = 0; r < MG_MAX_RANKS; ++r) {
      if (r >= po.world) break;
      if ((uint32_t)(wd[r][0] >> 32) != epoch || (uint32_t)(wd[r][1] >> 32) != epoch)
        wait_words(recv + (int64_t)r * po.slot, epoch, wd[r], t0, dead, r, po.timeout_ns);
      if (dead) break;
      const float rv = __uint_as_float((uint32_t)wd[r][0]);
      const int32_t ri = (int32_t)(uint32_t)wd[r][1];
      if (mg_argmax_better(rv, ri, best, bi)) {
        best = rv;
        bi = ri;
      }
    }
    idx[i] = bi == 0x7fffffff ? 0 : bi;
  }
  __syncthreads();  // every thread has read the count
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(po.count) = epoch;
}

}  // namespace

int mg_comm_peer_out(void* comm, PeerOut* out) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !out || !c->ready) return MG_ERR_INVALID_ARG;
  PeerOut po{};
  for (int r = 0; r < c->world; ++r) po.recv[r] = reinterpret_cast<uint64_t*>(c->peer[r]);
  po.count = reinterpret_cast<uint32_t*>(c->base + c->recv_bytes);
  po.done = po.count + 1;
  po.slot = c->slot;
  po.timeout_ns = c->timeout_ns;
  po.rank = c->rank;
  po.world = c->world;
  *out = po;
  return MG_OK;
}

extern "C" int mg_comm_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int mg_comm_create(int rank, int world, int64_t slot_elems, void** comm, void* ipc_handle) {
  if (!comm || !ipc_handle || world < 1 || world > MG_MAX_RANKS || rank < 0 || rank >= world || slot_elems <= 0)
    return MG_ERR_INVALID_ARG;
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  c->slot = ((slot_elems + 1) / 2 + 63) / 64 * 64;  // words of two values
  if (const char* v = getenv("MG_PEER_TIMEOUT_MS")) {
    const long long ms = atoll(v);
    if (ms > 0) c->timeout_ns = (uint64_t)ms * 1000000ull;
  }
  c->recv_bytes = align_up((size_t)2 * world * c->slot * sizeof(uint64_t), 256);
  c->bytes = c->recv_bytes + 256;  // + the two local counters
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->base), c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, c->bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->handle, c->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    delete c;
    return mg_set_cuda_error(e);
  }
  std::memcpy(ipc_handle, &c->handle, sizeof(cudaIpcMemHandle_t));
  *comm = c;
  return MG_OK;
}

extern "C" int mg_comm_open(void* comm, const void* ipc_handles) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !ipc_handles || c->ready) return MG_ERR_INVALID_ARG;
  const char* hs = static_cast<const char*>(ipc_handles);
  for (int r = 0; r < c->world; ++r) {
    const char* h = hs + (size_t)r * sizeof(cudaIpcMemHandle_t);
    if (r == c->rank || std::memcmp(h, &c->handle, sizeof(cudaIpcMemHandle_t)) == 0) {
      c->peer[r] = c->base;  // this rank's own area (a handle of this process maps to itself)
      continue;
    }
    cudaIpcMemHandle_t ph;
    std::memcpy(&ph, h, sizeof(ph));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ph, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return mg_set_cuda_error(e);
    c->peer[r] = static_cast<char*>(p);
    c->opened[r] = true;
  }
  c->ready = true;
  return MG_OK;
}

extern "C" int mg_comm_destroy(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return MG_ERR_INVALID_ARG;
  int rc = MG_OK;
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r] && cudaIpcCloseMemHandle(c->peer[r]) != cudaSuccess) rc = MG_ERR_CUDA;
  if (c->base && cudaFree(c->base) != cudaSuccess) rc = MG_ERR_CUDA;
  delete c;
  return rc;
}

extern "C" int mg_rowpar_reduce_norm(void* comm, float* h, const float* bias, int m, int n, int norm,
                                     const float* w, const float* wb, float eps, void* x, void* stream) {
  PeerOut po;
  int rc = mg_comm_peer_out(comm, &po);
  if (rc) return rc;
  if (!h || m < 0 || n <= 0 || n % 4 || n > 4 * kThreads * kMaxV || (int64_t)m * n > 2 * po.slot || norm < 0 ||
      norm > 2 || (norm && (!w || !x)) || (norm == 2 && !wb))
    return MG_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(wb) | reinterpret_cast<uintptr_t>(x)) & 15)
    return MG_ERR_INVALID_ARG;
  if (m == 0) return MG_OK;
  const int nv = n / 4;
  const int threads = nv >= kThreads ? kThreads : (nv + 31) / 32 * 32;
  MG_CUDA_TRY(mg_launch(rowpar_reduce_norm_kernel, dim3(m), dim3(threads), 0, mg_stream(stream), 1, po, h, bias,
                        n, norm, w, wb, eps, static_cast<__nv_bfloat16*>(x)));
  return MG_OK;
}

extern "C" int mg_vocab_argmax(void* comm, const float* logits, int m, int64_t n_local, int64_t ld, int64_t offset,
                               int32_t* idx, void* stream) {
  PeerOut po;
  int rc = mg_comm_peer_out(comm, &po);
  if (rc) return rc;
  if (!logits || !idx || m < 0 || m > 1024 || n_local <= 0 || ld < n_local || offset < 0 ||
      offset + n_local > 0x7fffffff || 2 * (int64_t)m > po.slot)
    return MG_ERR_INVALID_ARG;
  if (m == 0) return MG_OK;
  rc = mg_argmax_rows(logits, m, n_local, ld, idx, stream);
  if (rc) return rc;
  MG_CUDA_TRY(mg_launch(vocab_argmax_merge_kernel, dim3(1), dim3((unsigned)((m + 31) / 32 * 32)), 0,
                        mg_stream(stream), 1, po, logits, ld, n_local, offset, idx, m));
  return MG_OK;
}
