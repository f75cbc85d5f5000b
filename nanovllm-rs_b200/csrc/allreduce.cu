// Tensor-parallel epilogue: all-reduce of the row-parallel partial sums +
// residual add + RMSNorm in one kernel over NVLink peer memory.
//
// Replaces the NCCL all-reduce of RowParallelLinear::forward
// (nanovllm_rs/src/layers/linear.rs:200-208) and VocabParallelEmbedding
// (layers/embed_head.rs:58), made through AllReduce (layers/dist_util.rs:
// 29-84), fused with the RMSNorm that follows each of them in the decoder
// (models/qwen3.rs:232-238, 295; layers/layernorm.rs:18-42).
//
// Memory (one cudaMalloc per rank, opened by every peer through CUDA IPC):
//   in   [region]                    this rank's partial sums (the GEMM output)
//   recv [2 parities][world][region] partial rows pushed here by each peer
//   gath [2 parities][region]        reduced rows broadcast by their owners
//   flag [2][kArCtas][kMaxRanks] u32 barrier flags, written by peers
//   ep   [kArCtas] u32               per-CTA call epoch e (local only)
//
// One launch = kArCtas CTAs of 256 threads on every rank (a fixed grid, so
// the per-CTA epochs advance in lockstep whatever num_tokens is).  Row u of
// the batch belongs to CTA u % kArCtas on every rank, so every barrier pairs
// CTAs of the same index only.  Data moves by PUSH (peer stores of this
// rank's own rows), so no rank waits for another before it starts sending;
// each hand-off is a CTA barrier plus st.release.sys of flag = e in the
// receiver's memory, and the receiver's ld.acquire.sys spin.
//   one-shot (2 ranks): push every row to every peer's recv[e&1][rank];
//     hand-off; sum the world partials of each row (f32, rank order, one
//     rounding) and normalise it -- one hand-off, (n - 1) x the bytes out.
//   two-shot (3+ ranks): push row u to its owner o = u / ceil(T / n); hand-
//     off; the owner sums and pushes the reduced row into every rank's
//     gath[e&1]; hand-off; every rank normalises its rows from gath -- two
//     hand-offs, 2 (n - 1) / n x the bytes out.
// The sum feeds norm_row_load, the same code as nvkv_rms_norm.
// Buffer reuse: recv/gath alternate by epoch parity.  A peer can write the
// same parity again only two calls later, and it cannot finish the next call
// before this rank has entered it, i.e. finished reading this one; a rank's
// input is rewritten by its next GEMM, after this kernel, and is only read
// locally.
//
// Small messages (at most kArLLMaxBytes, e.g. a decode step's 256 x 4096
// rows) take the low-latency (LL) form instead: one-shot between two ranks;
// above, a column-owned two-shot (rank o owns a slice of every row's
// columns, so both phases spread over all CTAs -- a row-owned LL two-shot,
// whose owner phase ran on the few CTAs holding a rank's rows, measured
// slower than the flag hand-off at 8 ranks, 33.5 against 24.4 us per 2 MiB
// call, and was removed):
// every 8-byte word pushed to a peer carries 4 bytes of data and the call's
// epoch in its upper half, stored and polled as single-copy-atomic 64-bit
// words (st/ld.relaxed.sys).  The receiver spins on the words themselves, so
// there is no CTA barrier and no system-scope release between the pushes and
// the hand-off: a hand-off costs the data's flight time, at twice the bytes.
// Large messages keep the flag hand-off, whose fixed cost is small next to
// their transfer.  Both forms sum in the same order and give the same bits.
//   LL buffers: recv_ll [2 parities][world][ll_region]
//   (ll_region = 2 x the data bytes of kArLLMaxBytes).
//
// Every wait is bounded by the communicator's timeout (%globaltimer); on
// expiry the CTA records NVKV_DEVERR_PEER_TIMEOUT and returns.
#include <algorithm>
#include <cstring>
#include <new>

#include "norm_row.cuh"

namespace nvkv {

#ifndef NVKV_AR_CTAS
#define NVKV_AR_CTAS 148
#endif
constexpr int kArCtas = NVKV_AR_CTAS;  // CTAs per call (rows are dealt to them round-robin)
constexpr int kArMaxRanks = NVKV_COMM_MAX_RANKS;
constexpr size_t kArLLMaxBytes = (size_t)4 << 20;  // messages up to 4 MiB take the LL form

struct ArParams {
  uint8_t* base[kArMaxRanks];  // every rank's allocation (same layout)
  int64_t region;              // bytes of one [max_tokens, hidden] buffer slot
  int64_t off_recv, off_gath, off_flag;
  int64_t ll_region;           // bytes of one LL [rows, hidden] slot (2 x the data)
  int64_t off_recv_ll, off_gath_ll;
  uint32_t* epoch;             // this rank's per-CTA epochs
  int rank, world;
  int two_shot;
  int64_t T;
  int64_t S;  // rows per owner (two-shot)
  int H;
  void* residual;
  int res_mode;
  const void* w;
  float eps;
  void* out;
  int64_t timeout_ns;
  int* err;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Spins until *f has reached epoch e (wrap-safe); false after timeout_ns.
__device__ __forceinline__ bool wait_epoch(const uint32_t* f, uint32_t e, int64_t timeout_ns) {
  const uint64_t t0 = global_ns();
  for (uint32_t n = 1;; ++n) {
    if ((int32_t)(ld_acquire_sys(f) - e) >= 0) return true;
    if ((n & 63) == 0 && (int64_t)(global_ns() - t0) > timeout_ns) return false;
  }
}

// Addresses inside rank q's allocation.
__device__ __forceinline__ uint32_t* ar_flag(const ArParams& p, int q, int phase, int cta,
                                             int src) {
  return reinterpret_cast<uint32_t*>(p.base[q] + p.off_flag) +
         (phase * kArCtas + cta) * kArMaxRanks + src;
}
__device__ __forceinline__ uint8_t* ar_recv(const ArParams& p, int q, int par, int src,
                                            int64_t row) {
  return p.base[q] + p.off_recv + ((int64_t)par * p.world + src) * p.region +
         row * p.H * 2;
}
__device__ __forceinline__ uint8_t* ar_gath(const ArParams& p, int q, int par, int64_t row) {
  return p.base[q] + p.off_gath + (int64_t)par * p.region + row * p.H * 2;
}

// LL rows: 8-element vector c of a row (16 data bytes) is 4 words of 8 bytes,
// data in the low half, the epoch in the high half.
__device__ __forceinline__ uint8_t* ar_gath_ll(const ArParams& p, int q, int par, int64_t row) {
  return p.base[q] + p.off_gath_ll + (int64_t)par * p.ll_region + row * p.H * 4;
}
__device__ __forceinline__ uint8_t* ar_recv_ll(const ArParams& p, int q, int par, int src,
                                               int64_t row) {
  return p.base[q] + p.off_recv_ll + ((int64_t)par * p.world + src) * p.ll_region +
         row * p.H * 4;
}
// Pushes vector v (16 data bytes) as 4 LL words of epoch e at dst (32 bytes).
__device__ __forceinline__ void st_ll(uint8_t* dst, uint4 v, uint32_t e) {
  const uint64_t hi = (uint64_t)e << 32;
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(dst), "l"(hi | v.x),
               "l"(hi | v.y)
               : "memory");
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(dst + 16), "l"(hi | v.z),
               "l"(hi | v.w)
               : "memory");
}
// Polls the 4 LL words at src until all carry epoch e and returns their data;
// gives up (zeros, *fail set, error recorded once) after timeout_ns or as
// soon as another thread of the CTA has given up.
__device__ __forceinline__ uint4 ld_ll(const uint8_t* src, uint32_t e, int64_t timeout_ns,
                                       volatile int* fail, int* err) {
  uint64_t a, b, c, d;
  uint64_t t0 = 0;
  for (uint32_t n = 0;; ++n) {
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];"
                 : "=l"(a), "=l"(b)
                 : "l"(src)
                 : "memory");
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];"
                 : "=l"(c), "=l"(d)
                 : "l"(src + 16)
                 : "memory");
    if ((uint32_t)(a >> 32) == e && (uint32_t)(b >> 32) == e && (uint32_t)(c >> 32) == e &&
        (uint32_t)(d >> 32) == e)
      return make_uint4((uint32_t)a, (uint32_t)b, (uint32_t)c, (uint32_t)d);
    if ((n & 63) == 0) {
      if (n == 0) {
        t0 = global_ns();
      } else if (*fail || (int64_t)(global_ns() - t0) > timeout_ns) {
        if (!*fail) {
          *fail = 1;
          record_error(err, NVKV_DEVERR_PEER_TIMEOUT);
        }
        return make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
}

// dtype(sum over ranks, rank order) of 8-element vector c of a row whose
// per-rank partials are at src[q].
template <typename T>
__device__ __forceinline__ uint4 sum_vec(const uint8_t* const* src, int W, int c) {
  uint4 v[kArMaxRanks];
#pragma unroll
  for (int q = 0; q < kArMaxRanks; ++q)
    if (q < W) v[q] = __ldcg(reinterpret_cast<const uint4*>(src[q] + (int64_t)c * 16));
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
  for (int q = 0; q < kArMaxRanks; ++q) {
    if (q < W) {
      const uint32_t* vp = reinterpret_cast<const uint32_t*>(&v[q]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = DT<T>::to_f2(vp[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
  }
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int k = 0; k < 4; ++k) op[k] = DT<T>::from_f2(acc[2 * k], acc[2 * k + 1]);
  return o;
}

// CTA-uniform wait for flag (phase, cta, src) of this rank, src over the
// ranks in mask (bit q); false after the timeout (error recorded).
__device__ __forceinline__ bool ar_wait(const ArParams& p, int phase, int cta, uint32_t mask,
                                        uint32_t e, int* s_fail) {
  const int tid = threadIdx.x;
  if (tid < p.world && ((mask >> tid) & 1u) &&
      !wait_epoch(ar_flag(p, p.rank, phase, cta, tid), e, p.timeout_ns))
    *s_fail = 1;
  __syncthreads();
  if (*s_fail) {
    if (tid == 0) record_error(p.err, NVKV_DEVERR_PEER_TIMEOUT);
    return false;
  }
  return true;
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) allreduce_rms_norm_kernel(const ArParams p) {
  __shared__ float red[kNormThreads / 32];
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int W = p.world, r = p.rank, H = p.H, nvec = H / 8;
  const int64_t rb = (int64_t)H * 2;  // bytes per row
  if (tid == 0) {
    s_epoch = p.epoch[b] + 1;
    s_fail = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = (int)(e & 1u);
  const uint32_t peers = ((1u << W) - 1u) & ~(1u << r);
  const uint8_t* in = p.base[r];
  T* res = reinterpret_cast<T*>(p.residual);
  const T* wt = reinterpret_cast<const T*>(p.w);
  T* out = reinterpret_cast<T*>(p.out);

  if (!p.two_shot) {
    // ---- one-shot: push every row of this CTA to every peer ----
    for (int64_t u = b; u < p.T; u += kArCtas)
      for (int c = tid; c < nvec; c += kNormThreads) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(in + u * rb + (int64_t)c * 16));
#pragma unroll
        for (int q = 0; q < kArMaxRanks; ++q)
          if (q < W && q != r)
            *reinterpret_cast<uint4*>(ar_recv(p, q, par, r, u) + (int64_t)c * 16) = v;
      }
    // the barrier orders every thread's peer stores before the release
    // stores of the flags (cumulativity of st.release.sys)
    __syncthreads();
    if (tid < W && tid != r) st_release_sys(ar_flag(p, tid, 0, b, r), e);
    if (!ar_wait(p, 0, b, peers, e, &s_fail)) return;
    for (int64_t u = b; u < p.T; u += kArCtas) {
      const uint8_t* src[kArMaxRanks];
#pragma unroll
      for (int q = 0; q < kArMaxRanks; ++q)
        src[q] = q >= W ? nullptr : (q == r ? in + u * rb : ar_recv(p, r, par, q, u));
      T* ru = res + u * H;
      norm_row_load<T>([&](int c) { return sum_vec<T>(src, W, c); },
                       p.res_mode == NVKV_RESIDUAL_ADD ? ru : nullptr, ru, wt, p.eps,
                       out + u * H, H, red);
    }
  } else {
    // ---- two-shot: push each row to its owner, owners reduce and broadcast ----
    bool owns = false;
    for (int64_t u = b; u < p.T; u += kArCtas) {
      const int o = (int)(u / p.S);
      if (o == r) {
        owns = true;
        continue;
      }
      for (int c = tid; c < nvec; c += kNormThreads)
        *reinterpret_cast<uint4*>(ar_recv(p, o, par, r, u) + (int64_t)c * 16) =
            __ldcg(reinterpret_cast<const uint4*>(in + u * rb + (int64_t)c * 16));
    }
    __syncthreads();
    if (tid < W && tid != r) st_release_sys(ar_flag(p, tid, 0, b, r), e);
    if (owns) {
      if (!ar_wait(p, 0, b, peers, e, &s_fail)) return;
      for (int64_t u = b; u < p.T; u += kArCtas) {
        if ((int)(u / p.S) != r) continue;
        const uint8_t* src[kArMaxRanks];
#pragma unroll
        for (int q = 0; q < kArMaxRanks; ++q)
          src[q] = q >= W ? nullptr : (q == r ? in + u * rb : ar_recv(p, r, par, q, u));
        for (int c = tid; c < nvec; c += kNormThreads) {
          const uint4 s = sum_vec<T>(src, W, c);
#pragma unroll
          for (int q = 0; q < kArMaxRanks; ++q)
            if (q < W) *reinterpret_cast<uint4*>(ar_gath(p, q, par, u) + (int64_t)c * 16) = s;
        }
      }
    }
    __syncthreads();
    if (tid < W) st_release_sys(ar_flag(p, tid, 1, b, r), e);
    for (int64_t u = b; u < p.T; u += kArCtas) {
      if (!ar_wait(p, 1, b, 1u << (int)(u / p.S), e, &s_fail)) return;
      T* ru = res + u * H;
      norm_row<T>(reinterpret_cast<const T*>(ar_gath(p, r, par, u)),
                  p.res_mode == NVKV_RESIDUAL_ADD ? ru : nullptr, ru, wt, p.eps, out + u * H, H,
                  red);
    }
  }
  if (tid == 0) p.epoch[b] = e;
}

// f32 sum in rank order of 8-element vectors, rounded once (as sum_vec).
template <typename T>
__device__ __forceinline__ uint4 sum_vals(const uint4* v, int W) {
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
  for (int q = 0; q < kArMaxRanks; ++q) {
    if (q < W) {
      const uint32_t* vp = reinterpret_cast<const uint32_t*>(&v[q]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = DT<T>::to_f2(vp[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
  }
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int k = 0; k < 4; ++k) op[k] = DT<T>::from_f2(acc[2 * k], acc[2 * k + 1]);
  return o;
}

// The LL form of the kernel's one-shot protocol (same rows per CTA, same
// sums, same norm).
template <typename T>
__global__ void __launch_bounds__(kNormThreads) allreduce_rms_norm_ll_kernel(const ArParams p) {
  __shared__ float red[kNormThreads / 32];
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int W = p.world, r = p.rank, H = p.H, nvec = H / 8;
  const int64_t rb = (int64_t)H * 2;  // data bytes per row
  if (tid == 0) {
    s_epoch = p.epoch[b] + 1;
    s_fail = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = (int)(e & 1u);
  volatile int* fail = &s_fail;
  const uint8_t* in = p.base[r];
  T* res = reinterpret_cast<T*>(p.residual);
  const T* wt = reinterpret_cast<const T*>(p.w);
  T* out = reinterpret_cast<T*>(p.out);
  auto mine = [&](int64_t u, int c) {
    return __ldcg(reinterpret_cast<const uint4*>(in + u * rb + (int64_t)c * 16));
  };

  if (!p.two_shot) {
    // ---- one-shot: push every row of this CTA to every peer, sum on arrival ----
    for (int64_t u = b; u < p.T; u += kArCtas)
      for (int c = tid; c < nvec; c += kNormThreads) {
        const uint4 v = mine(u, c);
#pragma unroll
        for (int q = 0; q < kArMaxRanks; ++q)
          if (q < W && q != r) st_ll(ar_recv_ll(p, q, par, r, u) + (int64_t)c * 32, v, e);
      }
    for (int64_t u = b; u < p.T; u += kArCtas) {
      T* ru = res + u * H;
      norm_row_load<T>(
          [&](int c) {
            uint4 v[kArMaxRanks];
#pragma unroll
            for (int q = 0; q < kArMaxRanks; ++q)
              if (q < W)
                v[q] = q == r ? mine(u, c)
                              : ld_ll(ar_recv_ll(p, r, par, q, u) + (int64_t)c * 32, e,
                                      p.timeout_ns, fail, p.err);
            return sum_vals<T>(v, W);
          },
          p.res_mode == NVKV_RESIDUAL_ADD ? ru : nullptr, ru, wt, p.eps, out + u * H, H, red);
    }
  } else {
    // ---- two-shot, column-owned: rank o owns vectors [o nw, (o + 1) nw) of
    // every row.  Every CTA pushes each of its rows' slices to their owners,
    // sums the slice it owns over the ranks and pushes the sum to every rank,
    // then normalises its rows from the gathered sums: both phases spread
    // over all CTAs, each CTA exchanging with the CTAs of the same index ----
    const int nw = nvec / W;  // vectors per owner (the host checks nvec % W == 0)
    for (int64_t u = b; u < p.T; u += kArCtas)
      for (int c = tid; c < nvec; c += kNormThreads) {
        const int o = c / nw;
        if (o != r) st_ll(ar_recv_ll(p, o, par, r, u) + (int64_t)c * 32, mine(u, c), e);
      }
    for (int64_t u = b; u < p.T; u += kArCtas)
      for (int c = r * nw + tid; c < (r + 1) * nw; c += kNormThreads) {
        uint4 v[kArMaxRanks];
#pragma unroll
        for (int q = 0; q < kArMaxRanks; ++q)
          if (q < W)
            v[q] = q == r ? mine(u, c)
                          : ld_ll(ar_recv_ll(p, r, par, q, u) + (int64_t)c * 32, e, p.timeout_ns,
                                  fail, p.err);
        const uint4 sv = sum_vals<T>(v, W);
#pragma unroll
        for (int q = 0; q < kArMaxRanks; ++q)
          if (q < W) st_ll(ar_gath_ll(p, q, par, u) + (int64_t)c * 32, sv, e);
      }
    for (int64_t u = b; u < p.T; u += kArCtas) {
      T* ru = res + u * H;
      norm_row_load<T>(
          [&](int c) {
            return ld_ll(ar_gath_ll(p, r, par, u) + (int64_t)c * 32, e, p.timeout_ns, fail,
                         p.err);
          },
          p.res_mode == NVKV_RESIDUAL_ADD ? ru : nullptr, ru, wt, p.eps, out + u * H, H, red);
    }
  }
  __syncthreads();
  if (tid == 0 && !s_fail) p.epoch[b] = e;
}

}  // namespace nvkv

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct nvkv_comm {
  int rank = 0, world = 1, device = 0;
  size_t max_bytes = 0, region = 0;  // region: max_bytes rounded to 256
  uint8_t* base = nullptr;           // this rank's allocation
  uint8_t* peer[NVKV_COMM_MAX_RANKS] = {};
  bool opened = false;
  int64_t timeout_ns = 2000000000;
};

namespace nvkv {
namespace {

constexpr size_t kFlagBytes = 2 * kArCtas * kArMaxRanks * sizeof(uint32_t);
constexpr size_t kEpochBytes = kArCtas * sizeof(uint32_t);

size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }
// input | receive [2 parities][world sources] | gather [2 parities] | flags | epochs
size_t recv_off(const nvkv_comm* c) { return c->region; }
size_t gath_off(const nvkv_comm* c) { return c->region + 2 * (size_t)c->world * c->region; }
size_t flag_off(const nvkv_comm* c) { return gath_off(c) + 2 * c->region; }
size_t epoch_off(const nvkv_comm* c) { return flag_off(c) + round256(kFlagBytes); }
// LL slots hold 2 bytes of word per data byte, for messages up to kArLLMaxBytes
size_t ll_region(const nvkv_comm* c) { return 2 * std::min(c->region, kArLLMaxBytes); }
size_t recv_ll_off(const nvkv_comm* c) { return epoch_off(c) + round256(kEpochBytes); }
size_t gath_ll_off(const nvkv_comm* c) {
  return recv_ll_off(c) + 2 * (size_t)c->world * ll_region(c);
}
size_t total_bytes(const nvkv_comm* c) { return gath_ll_off(c) + 2 * ll_region(c); }

// One-shot (every rank pushes its whole partial to every peer, one barrier)
// for two ranks; two-shot (push to the row's owner, owner reduces and
// broadcasts, two barriers, 2 (n - 1) / n of the bytes) above.
// NVKV_AR_TWO_SHOT_MIN_RANKS moves the switch (tuning builds).
// LL form for the two-shot protocol too (column-owned).  Measured with the
// two-shot protocol forced at two ranks (2 MiB / 512 KiB / 128 KiB calls):
// 15.0 / 8.0 / 7.2 us against 18.5 / 15.2 / 14.3 for the flag hand-off and
// 15.2 / 7.9 / 6.3 for the one-shot LL form, bit-identical results.
#ifndef NVKV_AR_LL_TWO_SHOT
#define NVKV_AR_LL_TWO_SHOT 1
#endif
#ifndef NVKV_AR_TWO_SHOT_MIN_RANKS
#define NVKV_AR_TWO_SHOT_MIN_RANKS 3
#endif

static_assert(sizeof(cudaIpcMemHandle_t) <= NVKV_COMM_HANDLE_BYTES, "IPC handle size");

}  // namespace
}  // namespace nvkv

extern "C" int nvkv_comm_create(int rank, int world, size_t max_bytes, nvkv_comm_t* out,
                                void* handle_out) {
  using namespace nvkv;
  clear_error();
  if (!out || !handle_out) return set_error(NVKV_ERR_INVALID_ARG, "comm_create: null pointer");
  *out = nullptr;
  if (world < 1 || world > NVKV_COMM_MAX_RANKS || rank < 0 || rank >= world)
    return set_error(NVKV_ERR_INVALID_ARG, "comm_create: need 0 <= rank < world <= 8");
  if (max_bytes == 0 || max_bytes > ((size_t)1 << 34))
    return set_error(NVKV_ERR_INVALID_ARG, "comm_create: max_bytes must be in (0, 16 GiB]");
  nvkv_comm* c = new (std::nothrow) nvkv_comm;
  if (!c) return set_error(NVKV_ERR_CUDA, "comm_create: out of host memory");
  c->rank = rank;
  c->world = world;
  c->max_bytes = max_bytes;
  c->region = round256(max_bytes);
  int rc = check_cuda(cudaGetDevice(&c->device), "comm_create: cudaGetDevice");
  if (!rc) rc = check_cuda(cudaMalloc(&c->base, total_bytes(c)), "comm_create: cudaMalloc");
  if (!rc)
    rc = check_cuda(cudaMemset(c->base + flag_off(c), 0, total_bytes(c) - flag_off(c)),
                    "comm_create: zero flags");
  if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "comm_create: synchronize");
  cudaIpcMemHandle_t h;
  if (!rc) rc = check_cuda(cudaIpcGetMemHandle(&h, c->base), "comm_create: cudaIpcGetMemHandle");
  if (rc) {
    if (c->base) cudaFree(c->base);
    delete c;
    return rc;
  }
  std::memset(handle_out, 0, NVKV_COMM_HANDLE_BYTES);
  std::memcpy(handle_out, &h, sizeof(h));
  c->peer[rank] = c->base;
  *out = c;
  return NVKV_OK;
}

extern "C" int nvkv_comm_open_peers(nvkv_comm_t c, const void* handles) {
  using namespace nvkv;
  clear_error();
  if (!c || !handles) return set_error(NVKV_ERR_INVALID_ARG, "comm_open_peers: null pointer");
  if (c->opened) return set_error(NVKV_ERR_INVALID_ARG, "comm_open_peers: already open");
  int rc = check_cuda(cudaSetDevice(c->device), "comm_open_peers: cudaSetDevice");
  for (int q = 0; q < c->world && !rc; ++q) {
    if (q == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)q * NVKV_COMM_HANDLE_BYTES,
                sizeof(h));
    void* p = nullptr;
    rc = check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                    "comm_open_peers: cudaIpcOpenMemHandle");
    c->peer[q] = static_cast<uint8_t*>(p);
  }
  if (rc) {
    for (int q = 0; q < c->world; ++q)
      if (q != c->rank && c->peer[q]) {
        cudaIpcCloseMemHandle(c->peer[q]);
        c->peer[q] = nullptr;
      }
    return rc;
  }
  c->opened = true;
  return NVKV_OK;
}

extern "C" int nvkv_comm_input(nvkv_comm_t c, void** ptr) {
  using namespace nvkv;
  clear_error();
  if (!c || !ptr) return set_error(NVKV_ERR_INVALID_ARG, "comm_input: null pointer");
  *ptr = c->base;
  return NVKV_OK;
}

extern "C" int nvkv_comm_set_timeout(nvkv_comm_t c, int64_t timeout_ns) {
  using namespace nvkv;
  clear_error();
  if (!c || timeout_ns <= 0) return set_error(NVKV_ERR_INVALID_ARG, "comm_set_timeout: bad args");
  c->timeout_ns = timeout_ns;
  return NVKV_OK;
}

extern "C" int nvkv_comm_destroy(nvkv_comm_t c) {
  using namespace nvkv;
  clear_error();
  if (!c) return NVKV_OK;
  int rc = check_cuda(cudaSetDevice(c->device), "comm_destroy: cudaSetDevice");
  for (int q = 0; q < c->world; ++q)
    if (q != c->rank && c->peer[q]) {
      const int r2 = check_cuda(cudaIpcCloseMemHandle(c->peer[q]), "comm_destroy: close peer");
      if (!rc) rc = r2;
    }
  if (c->base) {
    const int r2 = check_cuda(cudaFree(c->base), "comm_destroy: cudaFree");
    if (!rc) rc = r2;
  }
  delete c;
  return rc;
}

extern "C" int nvkv_allreduce_rms_norm(nvkv_comm_t c, int64_t num_tokens, int hidden,
                                       void* residual, int residual_mode, const void* weight,
                                       float eps, void* out, int dtype, nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_allreduce_rms_norm");
  using namespace nvkv;
  clear_error();
  if (!c) return set_error(NVKV_ERR_INVALID_ARG, "allreduce_rms_norm: null comm");
  if (c->world > 1 && !c->opened)
    return set_error(NVKV_ERR_INVALID_ARG, "allreduce_rms_norm: peers not opened");
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "allreduce_rms_norm: unsupported dtype");
  if (hidden <= 0 || hidden % 8 != 0 || hidden > kNormThreads * 8 * kNormMaxVec)
    return set_error(NVKV_ERR_UNSUPPORTED,
                     "allreduce_rms_norm: hidden must be a multiple of 8, <= 8192");
  if (residual_mode != NVKV_RESIDUAL_ADD && residual_mode != NVKV_RESIDUAL_INIT)
    return set_error(NVKV_ERR_INVALID_ARG, "allreduce_rms_norm: bad residual_mode");
  if (num_tokens < 0) return set_error(NVKV_ERR_INVALID_ARG, "allreduce_rms_norm: negative size");
  if ((size_t)num_tokens * (size_t)hidden * 2 > c->max_bytes)
    return set_error(NVKV_ERR_INVALID_ARG, "allreduce_rms_norm: batch exceeds the comm buffer");
  // (an empty batch touches no buffer but still runs the barriers, so every
  // rank's epochs stay equal)
  if (num_tokens > 0 && (!residual || !weight || !out))
    return set_error(NVKV_ERR_INVALID_ARG, "allreduce_rms_norm: null pointer");
  if (!aligned16(residual) || !aligned16(weight) || !aligned16(out))
    return set_error(NVKV_ERR_ALIGNMENT, "allreduce_rms_norm: buffers must be 16-byte aligned");
  ArParams p;
  for (int q = 0; q < kArMaxRanks; ++q) p.base[q] = q < c->world ? c->peer[q] : nullptr;
  p.region = (int64_t)c->region;
  p.off_recv = (int64_t)recv_off(c);
  p.off_gath = (int64_t)gath_off(c);
  p.off_flag = (int64_t)flag_off(c);
  p.ll_region = (int64_t)ll_region(c);
  p.off_recv_ll = (int64_t)recv_ll_off(c);
  p.off_gath_ll = (int64_t)gath_ll_off(c);
  p.epoch = reinterpret_cast<uint32_t*>(c->base + epoch_off(c));
  p.rank = c->rank;
  p.world = c->world;
  p.two_shot = c->world >= NVKV_AR_TWO_SHOT_MIN_RANKS ? 1 : 0;
  p.T = num_tokens;
  p.S = (num_tokens + c->world - 1) / c->world;
  if (p.S == 0) p.S = 1;
  p.H = hidden;
  p.residual = residual;
  p.res_mode = residual_mode;
  p.w = weight;
  p.eps = eps;
  p.out = out;
  p.timeout_ns = c->timeout_ns;
  p.err = device_error_word();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // every rank sees the same num_tokens, so every rank takes the same form.
  // LL for the one-shot protocol (two ranks: 15.8 us per 2 MiB call, NCCL
  // 28.2) and for the column-owned two-shot one (NVKV_AR_LL_TWO_SHOT; the
  // hidden size's 8-element vectors must split evenly over the ranks).
  const bool small = (size_t)num_tokens * (size_t)hidden * 2 <= kArLLMaxBytes;
  const bool ll = small && (!p.two_shot || (NVKV_AR_LL_TWO_SHOT && (hidden / 8) % c->world == 0));
  if (dtype == NVKV_DTYPE_BF16) {
    if (ll)
      allreduce_rms_norm_ll_kernel<__nv_bfloat16><<<kArCtas, kNormThreads, 0, s>>>(p);
    else
      allreduce_rms_norm_kernel<__nv_bfloat16><<<kArCtas, kNormThreads, 0, s>>>(p);
  } else {
    if (ll)
      allreduce_rms_norm_ll_kernel<__half><<<kArCtas, kNormThreads, 0, s>>>(p);
    else
      allreduce_rms_norm_kernel<__half><<<kArCtas, kNormThreads, 0, s>>>(p);
  }
  return check_cuda(cudaGetLastError(), "allreduce_rms_norm launch");
}
