// Attention kernels (softmax(q k^T * scale + bottom-right causal mask) v).
//
// Semantics follow python/dli_ops/aot/attention/kernel.py:5-62: query row i of a
// sequence with Sq queries and Sk keys may see key j iff j <= i + (Sk - Sq)
// (kernel.py:35,49-50); scale defaults to 1/sqrt(D) (build_triton_aot_ops.py:283).
// GQA: query head h reads KV head h / (Hq / Hkv).
//
// All kernels are stride-generic: q/out element (b, h, s, d) lives at
// b*sb + h*sh + s*ss + d, and K/V rows of (b, kvh) are contiguous D-vectors at
// b*k_sb + kvh*k_sh + j*D. The key count of sequence b is `kv_len[b]` (a device
// array, so CUDA-graph replays can advance it) or the dense `seq_k`.
//
//  * cluster decode kernel (Sq * group <= 8 query rows per KV head): split-KV
//    flash decoding with keys on the MMA M side (S^T = K Q^T, O^T = V^T P^T),
//    the splits of one (sequence, KV head) merged inside a thread-block cluster
//    through distributed shared memory (no workspace, no combine launch).
//  * decode kernel (Sq * group <= 16 query rows per KV head): split-KV flash
//    decoding. CTA = (split, kv head, batch); the group's query rows form one
//    16-row MMA tile so each K/V byte fetched from HBM serves every query head
//    of the group. 4 warps each take 16 keys of every 64-key block
//    (cp.async 3-stage ring); partial (m, l, O) per split go to the workspace
//    and a combine kernel merges them.
//  * prefill kernel: FA2-style, CTA = (64 query rows, head, batch), 4 warps x
//    16 rows, 64-key blocks double-buffered with cp.async, QK^T and PV on
//    mma.sync m16n8k16 with fp32 accumulators, online softmax in registers.
//  * fallback kernel: exact fp32 (CUDA cores), any head_dim; serves fp32
//    graphs (the reference dtype) and head dims the MMA kernels do not cover.
#include <algorithm>
#include <cfloat>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "common.cuh"
#include "fmha.cuh"
#include "tcgen05.cuh"

namespace dli_sm100 {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxSplits = 16;  // split-KV partials merged per (sequence, KV head)
// K/V stages per decode CTA: 2 (3 CTAs per SM) or 3 (2 CTAs per SM).
static const int kDecodeStages = tuning_knob("ATTN_STAGES", 3) == 2 ? 2 : 3;

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t q_sb, q_sh, q_ss;
  int64_t o_sb, o_sh, o_ss;
  int64_t k_sb, k_sh;  // v uses the same strides
  int batch, hq, hkv, group, seq_q, seq_k, head_dim;
  const int64_t* positions;  // kv_len[b] = positions[b] + seq_q when non-null
  float scale_log2;          // scale * log2(e)
  int causal;                // 0: every key < kv_len is visible
  // split-KV decode
  int splits;
  float* part_o;    // [B, Hkv, splits, 16, D]
  float* part_ml;   // [B, Hkv, splits, 16, 2]
  unsigned* err;    // device error word (bounded waits, cache capacity)
};

__device__ __forceinline__ int kv_len_of(const AttnArgs& a, int b) {
  return a.positions ? static_cast<int>(a.positions[b]) + a.seq_q : a.seq_k;
}

// ---- MMA / ldmatrix / cp.async helpers ------------------------------------------
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Element offset of (row, col) inside a [rows x D] tile whose 16-byte chunks are
// XOR-swizzled by (row % 8) so ldmatrix row groups hit distinct banks.
template <int D>
__device__ __forceinline__ int swz(int row, int col) {
  return row * D + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7);
}

// Loads `rows` x D elements (row r of the tile = global row r0 + r, clipped to
// `limit` with zero fill) into a swizzled smem tile with 16-byte cp.async.
template <typename T, int D, int ROWS, int THREADS>
__device__ __forceinline__ void load_tile(T* smem_tile, const T* base, int r0, int limit) {
  constexpr int CPR = D / 8;  // 16-byte chunks per row
  const uint32_t s0 = static_cast<uint32_t>(__cvta_generic_to_shared(smem_tile));
  for (int c = threadIdx.x; c < ROWS * CPR; c += THREADS) {
    const int r = c / CPR, ch = c - r * CPR;
    const int gr = r0 + r;
    const bool valid = gr < limit;
    const T* src = base + static_cast<int64_t>(valid ? gr : 0) * D + ch * 8;
    cp_async16(s0 + swz<D>(r, ch * 8) * 2, src, valid);
  }
}

// ---- prefill ---------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(128)
    attn_prefill_kernel(const AttnArgs a) {
  DLI_PDL_ENTRY();
  constexpr int BM = 64, BN = 64;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* sq = reinterpret_cast<T*>(smem_raw);
  T* sk = sq + BM * D;          // [2][BN*D]
  T* sv = sk + 2 * BN * D;      // [2][BN*D]

  const int mb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / a.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int m0 = mb * BM;
  const int kv_len = kv_len_of(a, b);
  const int off = kv_len - a.seq_q;  // bottom-right causal offset
  const T* qbase = static_cast<const T*>(a.q) + b * a.q_sb + h * a.q_sh;
  const T* kbase = static_cast<const T*>(a.k) + b * a.k_sb + kvh * a.k_sh;
  const T* vbase = static_cast<const T*>(a.v) + b * a.k_sb + kvh * a.k_sh;

  // Q tile (rows may be strided: token-major layouts have q_ss != D).
  {
    constexpr int CPR = D / 8;
    const uint32_t s0 = static_cast<uint32_t>(__cvta_generic_to_shared(sq));
    for (int c = threadIdx.x; c < BM * CPR; c += 128) {
      const int r = c / CPR, ch = c - r * CPR;
      const int qs = m0 + r;
      const bool valid = qs < a.seq_q;
      cp_async16(s0 + swz<D>(r, ch * 8) * 2, qbase + (valid ? qs : 0) * a.q_ss + ch * 8, valid);
    }
  }
  int n_end = a.causal ? min(kv_len, m0 + BM + off) : kv_len;
  n_end = max(n_end, 0);
  const int nblocks = (n_end + BN - 1) / BN;
  if (nblocks > 0) {
    load_tile<T, D, BN, 128>(sk, kbase, 0, kv_len);
    load_tile<T, D, BN, 128>(sv, vbase, 0, kv_len);
  }
  cp_async_commit();

  uint32_t qf[D / 16][4];
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int qrow0 = m0 + warp * 16 + g;  // rows qrow0 and qrow0 + 8

  for (int nb = 0; nb < nblocks; ++nb) {
    const int buf = nb & 1;
    if (nb + 1 < nblocks) {
      load_tile<T, D, BN, 128>(sk + (buf ^ 1) * BN * D, kbase, (nb + 1) * BN, kv_len);
      load_tile<T, D, BN, 128>(sv + (buf ^ 1) * BN * D, vbase, (nb + 1) * BN, kv_len);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (nb == 0) {
      const uint32_t s0 = static_cast<uint32_t>(__cvta_generic_to_shared(sq));
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qf[kk], s0 + swz<D>(r, c) * 2);
      }
    }
    const T* kt = sk + buf * BN * D;
    const T* vt = sv + buf * BN * D;
    const uint32_t ks = static_cast<uint32_t>(__cvta_generic_to_shared(kt));
    const uint32_t vs = static_cast<uint32_t>(__cvta_generic_to_shared(vt));

    float s[BN / 8][4];
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
      for (int kk = 0; kk < D / 16; kk += 2) {
        uint32_t bf[4];
        const int r = nt * 8 + (lane & 7);
        const int c = kk * 16 + (lane >> 3) * 8;
        ldsm_x4(bf, ks + swz<D>(r, c) * 2);
        mma16816<T>(s[nt], qf[kk], bf[0], bf[1]);
        mma16816<T>(s[nt], qf[kk + 1], bf[2], bf[3]);
      }
    }
    // mask + online softmax
    const int n0 = nb * BN;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = n0 + nt * 8 + 2 * t + (e & 1);
        const int qr = qrow0 + (e >> 1) * 8;
        const bool vis = key < kv_len && (!a.causal || key <= qr + off);
        const float val = vis ? s[nt][e] * a.scale_log2 : -INFINITY;
        s[nt][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(mrow[r], mx[r]);
      alpha[r] = (mrow[r] == -INFINITY) ? 0.f : exp2f(mrow[r] - mnew);
      mrow[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mrow[e >> 1];
        const float p = (m == -INFINITY) ? 0.f : exp2f(s[nt][e] - m);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + rs[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        uint32_t bf[4];
        const int r = kk * 16 + (lane & 15);
        const int c = dt * 16 + (lane >> 4) * 8;
        ldsm_x4_t(bf, vs + swz<D>(r, c) * 2);
        mma16816<T>(o[2 * dt], pa, bf[0], bf[1]);
        mma16816<T>(o[2 * dt + 1], pa, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  T* obase = static_cast<T*>(a.out) + b * a.o_sb + h * a.o_sh;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qs = qrow0 + r * 8;
    if (qs >= a.seq_q) continue;
    const float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
    T* dst = obase + static_cast<int64_t>(qs) * a.o_ss;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int d = i * 8 + 2 * t;
      *reinterpret_cast<uint32_t*>(dst + d) = pack2<T>(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
    }
  }
}

// ---- decode (split-KV) ---------------------------------------------------------------
template <typename T, int D, int STAGES>
__global__ void __launch_bounds__(128, STAGES == 2 ? 3 : 2)
    attn_decode_kernel(const AttnArgs a) {
  DLI_PDL_ENTRY();
  constexpr int BN = 64;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* sk = reinterpret_cast<T*>(smem_raw);           // [STAGES][BN*D]
  T* sv = sk + STAGES * BN * D;                      // [STAGES][BN*D]
  float* so = reinterpret_cast<float*>(sv + STAGES * BN * D);  // [16][D] merged O
  float* sm = so + 16 * D;                           // [4][16] warp maxima
  float* sl = sm + 64;                               // [4][16] warp sums

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int kv_len = kv_len_of(a, b);
  const int off = kv_len - a.seq_q;
  const int rows = a.group * a.seq_q;  // <= 16
  // key range of this split, in whole 64-key blocks
  const int total_blocks = (kv_len + BN - 1) / BN;
  const int per_split = (total_blocks + a.splits - 1) / a.splits;
  const int blk0 = split * per_split;
  const int blk1 = min(blk0 + per_split, total_blocks);
  const int nblocks = max(blk1 - blk0, 0);

  const T* kbase = static_cast<const T*>(a.k) + b * a.k_sb + kvh * a.k_sh;
  const T* vbase = static_cast<const T*>(a.v) + b * a.k_sb + kvh * a.k_sh;

  // prologue loads
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) {
    if (st < nblocks) {
      load_tile<T, D, BN, 128>(sk + st * BN * D, kbase, (blk0 + st) * BN, kv_len);
      load_tile<T, D, BN, 128>(sv + st * BN * D, vbase, (blk0 + st) * BN, kv_len);
    }
    cp_async_commit();
  }

  // Q fragments straight from global: row r -> (s = r / group, head = kvh*group + r % group)
  uint32_t qf[D / 16][4];
  {
    const T* qb = static_cast<const T*>(a.q) + b * a.q_sb;
    auto qptr = [&](int r, int col) -> const T* {
      const int s = r / a.group, hh = kvh * a.group + (r - s * a.group);
      return qb + hh * a.q_sh + s * a.q_ss + col;
    };
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c0 = kk * 16 + 2 * t;
      uint32_t z = 0;
      qf[kk][0] = g < rows ? *reinterpret_cast<const uint32_t*>(qptr(g, c0)) : z;
      qf[kk][1] = g + 8 < rows ? *reinterpret_cast<const uint32_t*>(qptr(g + 8, c0)) : z;
      qf[kk][2] = g < rows ? *reinterpret_cast<const uint32_t*>(qptr(g, c0 + 8)) : z;
      qf[kk][3] = g + 8 < rows ? *reinterpret_cast<const uint32_t*>(qptr(g + 8, c0 + 8)) : z;
    }
  }
  // query token index of each of the thread's two rows (for the causal mask)
  const int qs0 = g < rows ? g / a.group : 0;
  const int qs1 = g + 8 < rows ? (g + 8) / a.group : 0;

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  for (int it = 0; it < nblocks; ++it) {
    const int pre = it + STAGES - 1;
    if (pre < nblocks) {
      const int st = pre % STAGES;
      load_tile<T, D, BN, 128>(sk + st * BN * D, kbase, (blk0 + pre) * BN, kv_len);
      load_tile<T, D, BN, 128>(sv + st * BN * D, vbase, (blk0 + pre) * BN, kv_len);
    }
    cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncthreads();
    const int st = it % STAGES;
    const uint32_t ks = static_cast<uint32_t>(__cvta_generic_to_shared(sk + st * BN * D));
    const uint32_t vs = static_cast<uint32_t>(__cvta_generic_to_shared(sv + st * BN * D));
    const int kw = warp * 16;  // this warp's 16 keys inside the block
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t bf[4];
      const int r = kw + (lane & 7) + ((lane >> 4) << 3);
      const int c = kk * 16 + ((lane >> 3) & 1) * 8;
      ldsm_x4(bf, ks + swz<D>(r, c) * 2);
      mma16816<T>(s[0], qf[kk], bf[0], bf[1]);
      mma16816<T>(s[1], qf[kk], bf[2], bf[3]);
    }
    const int n0 = (blk0 + it) * BN + kw;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = n0 + nt * 8 + 2 * t + (e & 1);
        const int qs = (e >> 1) ? qs1 : qs0;
        const bool vis = key < kv_len && (!a.causal || key <= qs + off);
        const float val = vis ? s[nt][e] * a.scale_log2 : -INFINITY;
        s[nt][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(mrow[r], mx[r]);
      alpha[r] = (mrow[r] == -INFINITY) ? 0.f : exp2f(mrow[r] - mnew);
      mrow[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mrow[e >> 1];
        const float p = (m == -INFINITY) ? 0.f : exp2f(s[nt][e] - m);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + rs[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    uint32_t pa[4];
    pa[0] = pack2<T>(s[0][0], s[0][1]);
    pa[1] = pack2<T>(s[0][2], s[0][3]);
    pa[2] = pack2<T>(s[1][0], s[1][1]);
    pa[3] = pack2<T>(s[1][2], s[1][3]);
#pragma unroll
    for (int dt = 0; dt < D / 16; ++dt) {
      uint32_t bf[4];
      const int r = kw + (lane & 15);
      const int c = dt * 16 + (lane >> 4) * 8;
      ldsm_x4_t(bf, vs + swz<D>(r, c) * 2);
      mma16816<T>(o[2 * dt], pa, bf[0], bf[1]);
      mma16816<T>(o[2 * dt + 1], pa, bf[2], bf[3]);
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // merge the 4 warps' states: row maxima / sums per warp, then scaled O sum
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  for (int i = threadIdx.x; i < 16 * D; i += 128) so[i] = 0.f;
  if (t == 0) {
    sm[warp * 16 + g] = mrow[0];
    sm[warp * 16 + g + 8] = mrow[1];
    sl[warp * 16 + g] = lrow[0];
    sl[warp * 16 + g + 8] = lrow[1];
  }
  __syncthreads();
  float mtot[2], ltot[2], scale[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g + 8 * r;
    float m = -INFINITY;
    for (int w = 0; w < 4; ++w) m = fmaxf(m, sm[w * 16 + row]);
    float l = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float mw = sm[w * 16 + row];
      l += (mw == -INFINITY) ? 0.f : sl[w * 16 + row] * exp2f(mw - m);
    }
    mtot[r] = m;
    ltot[r] = l;
    scale[r] = (mrow[r] == -INFINITY) ? 0.f : exp2f(mrow[r] - m);
  }
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int d = i * 8 + 2 * t;
    atomicAdd(&so[g * D + d], o[i][0] * scale[0]);
    atomicAdd(&so[g * D + d + 1], o[i][1] * scale[0]);
    atomicAdd(&so[(g + 8) * D + d], o[i][2] * scale[1]);
    atomicAdd(&so[(g + 8) * D + d + 1], o[i][3] * scale[1]);
  }
  __syncthreads();
  if (a.splits == 1) {
    // final output
    for (int i = threadIdx.x; i < rows * D; i += 128) {
      const int r = i / D, d = i - r * D;
      const int s = r / a.group, hh = kvh * a.group + (r - s * a.group);
      // every thread with this row computed identical mtot/ltot; recompute from smem
      float m = -INFINITY, l = 0.f;
      for (int w = 0; w < 4; ++w) m = fmaxf(m, sm[w * 16 + r]);
      for (int w = 0; w < 4; ++w) {
        const float mw = sm[w * 16 + r];
        l += (mw == -INFINITY) ? 0.f : sl[w * 16 + r] * exp2f(mw - m);
      }
      T* dst = static_cast<T*>(a.out) + b * a.o_sb + hh * a.o_sh + s * a.o_ss + d;
      *dst = from_f32<T>(l > 0.f ? so[r * D + d] / l : 0.f);
    }
  } else {
    const int64_t slot = ((static_cast<int64_t>(b) * a.hkv + kvh) * a.splits + split);
    float* po = a.part_o + slot * 16 * D;
    for (int i = threadIdx.x; i < 16 * D; i += 128) po[i] = so[i];
    if (t == 0 && warp == 0) {
      float* pml = a.part_ml + slot * 32;
      pml[g * 2] = mtot[0];
      pml[g * 2 + 1] = ltot[0];
      pml[(g + 8) * 2] = mtot[1];
      pml[(g + 8) * 2 + 1] = ltot[1];
    }
  }
}

// ---- decode with keys on the MMA M side, split-KV reduced inside a cluster ----------
// For up to 8 query rows per KV head (decode: the GQA group of one token).
// S^T = K Q^T puts 16 keys on the m16 side and the <= 8 query rows on n8, so a
// 7-head group wastes 1/8 of the tensor work instead of 9/16 with a 16-row
// query tile, and each thread keeps 2 rows' softmax state and a D x 8 O^T
// accumulator (32 registers at D = 128). P^T for O^T += V^T P^T is the
// transpose of the S^T fragment: movmatrix turns the accumulator layout into
// the B-operand layout without shared memory. The S splits of one (sequence,
// KV head) form a thread-block cluster; their (m, l, O) states are merged
// through distributed shared memory in rank order (deterministic), so the
// kernel needs no workspace and no combine launch.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ void ldsm_x4_a(uint32_t (&r)[4], uint32_t addr) { ldsm_x4(r, addr); }

// TMA: K/V blocks arrive by tensor-map copies (one elected thread, per-stage
// full/empty mbarriers, no CTA barrier inside the key loop) into D/64 boxes of
// [64 keys][64 elements] with the 128-byte swizzle; otherwise every thread
// issues 16-byte cp.async into row-major swizzled tiles.
template <typename T, int D, int STAGES, bool TMA>
struct DecodeClusterSmem {
  static constexpr int kRing = 2 * STAGES * 64 * D * 2;     // K and V stages
  static constexpr int kQ = 8 * D * 2;                      // swizzled Q rows
  static constexpr int kWarpO = 4 * 8 * D * 4;              // per-warp scaled O^T (aliases the ring)
  static constexpr int kState = 8 * D * 4 + 2 * 8 * 4;      // merged O [8][D], m[8], l[8]
  static constexpr int kWarpML = 2 * 4 * 8 * 4;             // per-warp m, l
  static constexpr int kBarOff = kRing + kQ + kState + kWarpML;
  static constexpr int kBars = TMA ? 2 * STAGES * 8 : 0;   // full[STAGES], empty[STAGES]
  static constexpr int kSlack = TMA ? 1024 : 0;             // ring base rounded up to 1 KiB
  static constexpr int kBytes = kBarOff + kBars + kSlack;
  static_assert(kWarpO <= kRing, "warp partials alias the K/V ring");
  static_assert(kBarOff % 8 == 0, "mbarrier alignment");
};

// Element offset of (key row, column) in one K or V stage.
template <int D, bool TMA>
__device__ __forceinline__ int kv_swz(int row, int col) {
  if constexpr (TMA)
    return (col >> 6) * (64 * 64) + row * 64 + ((((col >> 3) & 7) ^ (row & 7)) << 3) + (col & 7);
  else
    return swz<D>(row, col);
}

template <typename T, int D, int STAGES, bool TMA>
__global__ void __launch_bounds__(128)
    attn_decode_cluster_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap tk,
                               const __grid_constant__ CUtensorMap tv) {
  DLI_PDL_ENTRY();
  using L = DecodeClusterSmem<T, D, STAGES, TMA>;
  constexpr int BN = 64;
  extern __shared__ __align__(16) uint8_t smem_base[];
  // the same offset in every CTA of the launch, so DSMEM addresses still map rank to rank
  uint8_t* smem_raw = TMA ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_base) + 1023) &
                                                       ~static_cast<uintptr_t>(1023))
                          : smem_base;
  T* sk = reinterpret_cast<T*>(smem_raw);                       // [STAGES][BN*D]
  T* sv = sk + STAGES * BN * D;                                  // [STAGES][BN*D]
  T* sq = reinterpret_cast<T*>(smem_raw + L::kRing);            // [8][D] swizzled
  float* co = reinterpret_cast<float*>(smem_raw + L::kRing + L::kQ);  // merged O [8][D]
  float* cm = co + 8 * D;                                        // merged m [8]
  float* cl = cm + 8;                                            // merged l [8]
  float* wm = cl + 8;                                            // [4][8]
  float* wl = wm + 32;                                           // [4][8]
  float* wo = reinterpret_cast<float*>(smem_raw);                // [4][8][D], after the loop

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nsplit = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  int kv_len = kv_len_of(a, b);
  if constexpr (TMA) {
    const int64_t cap = a.k_sh / D;  // cache rows per head (the tensor maps' row extent)
    if (kv_len > cap) {
      if (threadIdx.x == 0) set_device_error(a.err, kDevErrKvCapacity);
      kv_len = static_cast<int>(cap);
    }
  }
  const int off = kv_len - a.seq_q;
  const int rows = a.group * a.seq_q;  // <= 8
  const int total_blocks = (kv_len + BN - 1) / BN;
  const int blk0 = static_cast<int>(static_cast<int64_t>(split) * total_blocks / nsplit);
  const int blk1 = static_cast<int>(static_cast<int64_t>(split + 1) * total_blocks / nsplit);
  const int nblocks = blk1 - blk0;

  const T* kbase = static_cast<const T*>(a.k) + b * a.k_sb + kvh * a.k_sh;
  const T* vbase = static_cast<const T*>(a.v) + b * a.k_sb + kvh * a.k_sh;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + L::kBarOff);  // TMA only
  uint64_t* empty = full + STAGES;
  // K and V of block j (of this split) into stage st, completing on full[st]
  auto issue_kv = [&](int j, int st) {
    mbar_arrive_expect_tx(&full[st], 2 * BN * D * 2);
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
      tma_load_4d(sk + st * BN * D + c * 64 * 64, &tk, c * 64, (blk0 + j) * BN, kvh, b, &full[st]);
      tma_load_4d(sv + st * BN * D + c * 64 * 64, &tv, c * 64, (blk0 + j) * BN, kvh, b, &full[st]);
    }
  };
  int issued = 0;      // thread 0: K/V blocks issued by TMA
  bool refill = true;  // thread 0: cleared when a stage was never released
  if constexpr (TMA) {
    if (threadIdx.x == 0) {
      for (int st = 0; st < STAGES; ++st) {
        mbar_init(&full[st], 1);
        mbar_init(&empty[st], 4);  // one arrival per warp
      }
      mbar_fence_init();
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      for (; issued < STAGES && issued < nblocks; ++issued) issue_kv(issued, issued);
    }
  }

  // Q rows r -> (token s = r / group, head kvh*group + r % group); rows >= `rows` zero
  {
    const T* qb = static_cast<const T*>(a.q) + b * a.q_sb;
    const uint32_t s0 = static_cast<uint32_t>(__cvta_generic_to_shared(sq));
    for (int c = threadIdx.x; c < 8 * (D / 8); c += 128) {
      const int r = c / (D / 8), ch = c - r * (D / 8);
      const bool valid = r < rows;
      const int qs = valid ? r / a.group : 0, hh = kvh * a.group + (valid ? r - qs * a.group : 0);
      cp_async16(s0 + swz<D>(r, ch * 8) * 2, qb + hh * a.q_sh + qs * a.q_ss + ch * 8, valid);
    }
  }
  if constexpr (TMA) {
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();  // Q and the initialised barriers are visible to every warp
  } else {
#pragma unroll
    for (int st = 0; st < STAGES - 1; ++st) {
      if (st < nblocks) {
        load_tile<T, D, BN, 128>(sk + st * BN * D, kbase, (blk0 + st) * BN, kv_len);
        load_tile<T, D, BN, 128>(sv + st * BN * D, vbase, (blk0 + st) * BN, kv_len);
      }
      cp_async_commit();  // the first group also carries Q
    }
  }

  // query token of the thread's two score columns (rows 2t, 2t+1), for the causal mask
  const int qs0 = (2 * t) < rows ? (2 * t) / a.group : 0;
  const int qs1 = (2 * t + 1) < rows ? (2 * t + 1) / a.group : 0;

  uint32_t qf[D / 16][2];
  float o[D / 16][4];
#pragma unroll
  for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int kw = warp * 16;  // this warp's 16 keys of every block

  for (int it = 0; it < nblocks; ++it) {
    if constexpr (TMA) {
      // every lane observes the phase, then the warp agrees (uniform exit)
      const bool got = mbar_wait(&full[it % STAGES], (it / STAGES) & 1);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) set_device_error(a.err, kDevErrAttentionTimeout);
        break;
      }
    } else {
      const int pre = it + STAGES - 1;
      if (pre < nblocks) {
        const int st = pre % STAGES;
        load_tile<T, D, BN, 128>(sk + st * BN * D, kbase, (blk0 + pre) * BN, kv_len);
        load_tile<T, D, BN, 128>(sv + st * BN * D, vbase, (blk0 + pre) * BN, kv_len);
      }
      cp_async_commit();
      cp_async_wait<STAGES - 1>();
      __syncthreads();
    }
    if (it == 0) {
      // Q^T B fragments: ldmatrix of the [8 rows][16 dims] slices
      const uint32_t qa = static_cast<uint32_t>(__cvta_generic_to_shared(sq));
#pragma unroll
      for (int kk = 0; kk < D / 16; kk += 2) {
        uint32_t r4[4];
        ldsm_x4(r4, qa + swz<D>(lane & 7, kk * 16 + (lane >> 3) * 8) * 2);
        qf[kk][0] = r4[0];
        qf[kk][1] = r4[1];
        qf[kk + 1][0] = r4[2];
        qf[kk + 1][1] = r4[3];
      }
    }
    const int st = it % STAGES;
    const uint32_t ks = static_cast<uint32_t>(__cvta_generic_to_shared(sk + st * BN * D));
    const uint32_t vs = static_cast<uint32_t>(__cvta_generic_to_shared(sv + st * BN * D));

    // S^T [16 keys x 8 rows]
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t af[4];
      ldsm_x4_a(af, ks + kv_swz<D, TMA>(kw + (lane & 7) + ((lane >> 3) & 1) * 8, kk * 16 + (lane >> 4) * 8) * 2);
      mma16816<T>(sc, af, qf[kk][0], qf[kk][1]);
    }
    const int key0 = (blk0 + it) * BN + kw + g, key1 = key0 + 8;
    const bool v00 = key0 < kv_len && (!a.causal || key0 <= qs0 + off);
    const bool v01 = key0 < kv_len && (!a.causal || key0 <= qs1 + off);
    const bool v10 = key1 < kv_len && (!a.causal || key1 <= qs0 + off);
    const bool v11 = key1 < kv_len && (!a.causal || key1 <= qs1 + off);
    const float s00 = v00 ? sc[0] * a.scale_log2 : -INFINITY;  // key0, row 2t
    const float s01 = v01 ? sc[1] * a.scale_log2 : -INFINITY;  // key0, row 2t+1
    const float s10 = v10 ? sc[2] * a.scale_log2 : -INFINITY;  // key1, row 2t
    const float s11 = v11 ? sc[3] * a.scale_log2 : -INFINITY;  // key1, row 2t+1
    float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
    for (int sh = 4; sh < 32; sh <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
    }
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float al0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - n0);
    const float al1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - n1);
    m0 = n0;
    m1 = n1;
    const float p00 = (n0 == -INFINITY) ? 0.f : exp2f(s00 - n0);
    const float p10 = (n0 == -INFINITY) ? 0.f : exp2f(s10 - n0);
    const float p01 = (n1 == -INFINITY) ? 0.f : exp2f(s01 - n1);
    const float p11 = (n1 == -INFINITY) ? 0.f : exp2f(s11 - n1);
    l0 = l0 * al0 + p00 + p10;  // this thread's keys; summed over the warp at the end
    l1 = l1 * al1 + p01 + p11;
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      o[i][0] *= al0;
      o[i][1] *= al1;
      o[i][2] *= al0;
      o[i][3] *= al1;
    }
    // P^T as the B operand: transpose the two 8x8 accumulator blocks
    const uint32_t pb0 = movmatrix_t(pack2<T>(p00, p01));
    const uint32_t pb1 = movmatrix_t(pack2<T>(p10, p11));
    if constexpr (TMA) {
      // V rows of keys >= kv_len hold whatever the cache had there (the copy
      // is not clipped to the sequence): zero this warp's rows so a stale
      // non-finite value cannot reach O through a zero weight
      const int kfirst = (blk0 + it) * BN + kw;
      if (kfirst + 16 > kv_len) {
        T* vt = sv + (it % STAGES) * BN * D;
        for (int c = lane; c < 16 * (D / 8); c += 32) {
          const int r = c / (D / 8), ch = c - r * (D / 8);
          if (kfirst + r >= kv_len)
            *reinterpret_cast<uint4*>(vt + kv_swz<D, TMA>(kw + r, ch * 8)) = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
    }
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      uint32_t va[4];
      ldsm_x4_t(va, vs + kv_swz<D, TMA>(kw + (lane & 7) + (lane >> 4) * 8, mt * 16 + ((lane >> 3) & 1) * 8) * 2);
      mma16816<T>(o[mt], va, pb0, pb1);
    }
    if constexpr (TMA) {
      const int st = it % STAGES;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
      if (threadIdx.x == 0 && refill && issued < nblocks) {
        // refill the stage once all four warps have released it
        if (mbar_wait(&empty[st], (it / STAGES) & 1)) {
          issue_kv(issued, st);
          ++issued;
        } else {
          set_device_error(a.err, kDevErrAttentionTimeout);
          refill = false;
        }
      }
      __syncwarp();
    } else {
      __syncthreads();
    }
  }
  if constexpr (TMA) {
    // no copy may still be writing the ring when it becomes the partial area
    if (threadIdx.x == 0)
      for (int j = max(0, issued - STAGES); j < issued; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1);
  } else {
    cp_async_wait<0>();
  }
  __syncthreads();  // the ring becomes the warp-partial area

  // merge the 4 warps (fixed order)
#pragma unroll
  for (int sh = 4; sh < 32; sh <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
    l1 += __shfl_xor_sync(0xffffffffu, l1, sh);
  }
  if (g == 0) {
    wm[warp * 8 + 2 * t] = m0;
    wm[warp * 8 + 2 * t + 1] = m1;
    wl[warp * 8 + 2 * t] = l0;
    wl[warp * 8 + 2 * t + 1] = l1;
  }
  __syncthreads();
  {
    float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      M0 = fmaxf(M0, wm[w * 8 + 2 * t]);
      M1 = fmaxf(M1, wm[w * 8 + 2 * t + 1]);
    }
    const float f0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - M0);
    const float f1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - M1);
    float* myo = wo + warp * 8 * D;
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int d = mt * 16 + g;
      myo[(2 * t) * D + d] = o[mt][0] * f0;
      myo[(2 * t + 1) * D + d] = o[mt][1] * f1;
      myo[(2 * t) * D + d + 8] = o[mt][2] * f0;
      myo[(2 * t + 1) * D + d + 8] = o[mt][3] * f1;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 8 * D; i += 128) {
    co[i] = ((wo[i] + wo[8 * D + i]) + wo[2 * 8 * D + i]) + wo[3 * 8 * D + i];
  }
  if (threadIdx.x < 8) {
    const int r = threadIdx.x;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w * 8 + r]);
    float Lsum = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = wm[w * 8 + r];
      Lsum += (mw == -INFINITY) ? 0.f : wl[w * 8 + r] * exp2f(mw - M);
    }
    cm[r] = M;
    cl[r] = Lsum;
  }
  if (nsplit == 1) {
    __syncthreads();
    for (int i = threadIdx.x; i < rows * D; i += 128) {
      const int r = i / D, d = i - r * D;
      const int qs = r / a.group, hh = kvh * a.group + (r - qs * a.group);
      T* dst = static_cast<T*>(a.out) + b * a.o_sb + hh * a.o_sh + qs * a.o_ss + d;
      *dst = from_f32<T>(cl[r] > 0.f ? co[r * D + d] / cl[r] : 0.f);
    }
    return;
  }
  // merge the cluster's splits: rank r writes every nsplit-th quad of the output
  cluster_sync();
  const uint32_t co_local = static_cast<uint32_t>(__cvta_generic_to_shared(co));
  const uint32_t cm_local = static_cast<uint32_t>(__cvta_generic_to_shared(cm));
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int quads = rows * (D / 4);
  for (int q = static_cast<int>(rank) * 128 + threadIdx.x; q < quads; q += nsplit * 128) {
    const int r = q / (D / 4), d = (q - r * (D / 4)) * 4;
    // every rank's (m, l, O quad) is requested before any is used: one DSMEM round trip
    float ms[8], ls[8];
    float4 ov[8];
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) {
      if (s2 < nsplit) {
        const uint32_t base = mapa_shared(cm_local, static_cast<uint32_t>(s2));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ms[s2]) : "r"(base + r * 4) : "memory");
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ls[s2]) : "r"(base + (8 + r) * 4) : "memory");
        ov[s2] = ld_dsmem_f4(mapa_shared(co_local + (r * D + d) * 4, static_cast<uint32_t>(s2)));
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2)
      if (s2 < nsplit) M = fmaxf(M, ms[s2]);
    float Lsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) {
      if (s2 >= nsplit || ms[s2] == -INFINITY) continue;
      const float w = exp2f(ms[s2] - M);
      Lsum += ls[s2] * w;
      acc.x += ov[s2].x * w;
      acc.y += ov[s2].y * w;
      acc.z += ov[s2].z * w;
      acc.w += ov[s2].w * w;
    }
    const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
    const int qs = r / a.group, hh = kvh * a.group + (r - qs * a.group);
    T* dst = static_cast<T*>(a.out) + b * a.o_sb + hh * a.o_sh + qs * a.o_ss + d;
    dst[0] = from_f32<T>(acc.x * inv);
    dst[1] = from_f32<T>(acc.y * inv);
    dst[2] = from_f32<T>(acc.z * inv);
    dst[3] = from_f32<T>(acc.w * inv);
  }
  cluster_sync();  // keep this CTA's state alive until every rank has read it
}

// Merges split partials: out = sum_s O_s 2^(m_s - M) / sum_s l_s 2^(m_s - M).
template <typename T>
__global__ void attn_combine_kernel(const AttnArgs a) {
  DLI_PDL_ENTRY();
  // One thread per (query row, 4 dims); every split's (m, l) and O quad are
  // fetched with independent loads (splits <= kMaxSplits, unrolled) so the
  // merge costs two memory round trips.
  const int kvh = blockIdx.x, b = blockIdx.y;
  const int rows = a.group * a.seq_q;
  const int D = a.head_dim;
  const int quads = D / 4;
  const int64_t slot0 = (static_cast<int64_t>(b) * a.hkv + kvh) * a.splits;
  for (int i = threadIdx.x; i < rows * quads; i += blockDim.x) {
    const int r = i / quads, d = (i - r * quads) * 4;
    float ms[kMaxSplits];
    float m = -INFINITY;
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s) {
      ms[s] = s < a.splits ? a.part_ml[(slot0 + s) * 32 + r * 2] : -INFINITY;
      m = fmaxf(m, ms[s]);
    }
    float l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s) {
      if (s >= a.splits || ms[s] == -INFINITY) continue;
      const float w = exp2f(ms[s] - m);
      l += a.part_ml[(slot0 + s) * 32 + r * 2 + 1] * w;
      const float4 o = *reinterpret_cast<const float4*>(a.part_o + (slot0 + s) * 16 * D + r * D + d);
      acc.x += o.x * w;
      acc.y += o.y * w;
      acc.z += o.z * w;
      acc.w += o.w * w;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int sq = r / a.group, hh = kvh * a.group + (r - sq * a.group);
    T* dst = static_cast<T*>(a.out) + b * a.o_sb + hh * a.o_sh + sq * a.o_ss + d;
    dst[0] = from_f32<T>(acc.x * inv);
    dst[1] = from_f32<T>(acc.y * inv);
    dst[2] = from_f32<T>(acc.z * inv);
    dst[3] = from_f32<T>(acc.w * inv);
  }
}

// ---- exact fp32 fallback ---------------------------------------------------------------
// One warp per query row; lanes split the keys of each 32-key chunk (dot products
// read q from shared memory), then the chunk's probabilities are broadcast and
// each lane accumulates its own dims of O. Exact fp32 math with expf.
template <typename T>
__global__ void attn_fallback_kernel(const AttnArgs a) {
  DLI_PDL_ENTRY();
  extern __shared__ float sqf[];  // [warps][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * nwarps + warp;
  const int64_t total = static_cast<int64_t>(a.batch) * a.hq * a.seq_q;
  if (row >= total) return;
  const int qs = static_cast<int>(row % a.seq_q);
  const int h = static_cast<int>((row / a.seq_q) % a.hq);
  const int b = static_cast<int>(row / (static_cast<int64_t>(a.seq_q) * a.hq));
  const int kvh = h / a.group;
  const int D = a.head_dim;
  const int kv_len = kv_len_of(a, b);
  const int off = kv_len - a.seq_q;
  const float scale = a.scale_log2 / kLog2e;
  float* qv = sqf + warp * D;
  const T* qp = static_cast<const T*>(a.q) + b * a.q_sb + h * a.q_sh + qs * a.q_ss;
  for (int d = lane; d < D; d += 32) qv[d] = to_f32(qp[d]);
  __syncwarp();
  const T* kb = static_cast<const T*>(a.k) + b * a.k_sb + kvh * a.k_sh;
  const T* vb = static_cast<const T*>(a.v) + b * a.k_sb + kvh * a.k_sh;
  const int nkeys = a.causal ? max(0, min(kv_len, qs + off + 1)) : kv_len;
  float m = -INFINITY, l = 0.f;
  float acc[8];  // dims lane, lane+32, ... (D <= 256)
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int j0 = 0; j0 < nkeys; j0 += 32) {
    const int j = j0 + lane;
    float sc = -INFINITY;
    if (j < nkeys) {
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(qv[d], to_f32(kb[static_cast<int64_t>(j) * D + d]), dot);
      sc = dot * scale;
    }
    const float cm = warp_max(sc);
    const float mnew = fmaxf(m, cm);
    const float alpha = (m == -INFINITY) ? 0.f : expf(m - mnew);
    const float p = (sc == -INFINITY) ? 0.f : expf(sc - mnew);
    l = l * alpha + warp_sum(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= alpha;
    const int cnt = min(32, nkeys - j0);
    for (int jj = 0; jj < cnt; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const T* vr = vb + static_cast<int64_t>(j0 + jj) * D;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] = fmaf(pj, to_f32(vr[d]), acc[i]);
      }
    }
    m = mnew;
  }
  T* op = static_cast<T*>(a.out) + b * a.o_sb + h * a.o_sh + qs * a.o_ss;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < D) op[d] = from_f32<T>(l > 0.f ? acc[i] / l : 0.f);
  }
}

// ---- fp32 tiles on CUDA cores (the reference's dtype) -------------------------------------
// CTA = W·RW query rows of one (sequence, query head) x one split of the keys;
// W warps of RW rows each (RW = 8 by default, 4 with DLI_SM100_ATTN_F32_RW=4;
// W = 8 by default, 4 with DLI_SM100_ATTN_F32_WARPS=4). Eight warps give 16
// warps per SM (two 110 KB CTAs); the kernel is bound by instruction latency, and
// at B·H = 896, 128 x 128 causal tiles, D = 128 it takes 216 us against 249 us
// with four warps and 319 us with four warps of four rows.
// 32-key K/V blocks are double-buffered in shared memory with cp.async.
//  * S = Q K^T, RW = 8: lane (g, c) = (lane / 8, lane % 8) scores rows 2g, 2g+1 of
//    the warp against keys c, c+8, c+16, c+24 of the block. Per 4-wide d step a
//    lane reads 2 Q and 4 K float4s for 32 FMAs (Q and K rows padded by 4 floats),
//    where one key per lane against 8 broadcast rows read 9. The row max and sum
//    reduce over the 8 lanes of a group (3 shuffles) and reach the other lanes by
//    one shuffle per row, where a whole-warp reduction per row took 5. Measured at
//    B·H 896, 128 x 128: shared loads 13.8 M -> 10.3 M instructions at the same
//    32.3 M wavefronts, 217 -> 195 us.
//    RW = 4: lane j scores key j against the warp's 4 rows, max and sum reduce
//    over the warp.
//  * The online softmax state (m, l) of every row of the warp is held by every
//    lane.
//  * O += P V: each lane owns D/32 output columns. The warp's probabilities go
//    through a small per-warp tile in shared memory ([32 keys][RW], written as
//    float4s on conflict-free padded rows) and come back as broadcast float4s:
//    per key one V read and RW/4 broadcasts feed RW·D/32 FMAs per lane, where a
//    shuffle per (row, key) would bound the loop on the shuffle unit.
//  * A warp whose rows cannot see any key of a block (causal) skips it: the
//    skipped update would have been exact (alpha = 1, p = 0).
// When the rows alone cannot fill the GPU (decode), the keys are split over up to
// 8 CTAs of a thread-block cluster whose (m, l, O) are merged through distributed
// shared memory in rank order, in the freed K/V stages: exact fp32, deterministic,
// no workspace. Rows past a sequence's keys are never loaded (cp.async zero-fills
// them). The launch shape (W, RW) changes where rows are split and the order in
// which a block's probabilities are summed, both within fp32 rounding.
constexpr int kF32Keys = 32;

template <int D, int RW, int W>
struct F32AttnSmem {
  static_assert(RW == 4 || RW == 8, "4 or 8 query rows per warp");
  static_assert(W == 4 || W == 8, "4 or 8 warps");
  static constexpr int kThreads = 32 * W;
  static constexpr int kRows = W * RW;                 // query rows per CTA
  static constexpr int kRow = D + 4;                   // padded K/V row (floats)
  static constexpr int kPRow = RW == 8 ? 12 : 4;       // padded P row of one key (floats)
  static constexpr int kQRow = D + 4;                  // padded Q row (floats)
  static constexpr int kQ = kRows * kQRow;             // [kRows][D+4]
  static constexpr int kKV = 2 * 2 * kF32Keys * kRow;  // 2 stages x (K, V) x [32][D+4]
  static constexpr int kP = W * kF32Keys * kPRow;      // per warp [32 keys][kPRow]
  static constexpr int kState = kRows * (D + 2);       // merge: O [kRows][D] + m, l per row
  static_assert(kState <= kKV, "the merge state reuses the K/V stages");
  static constexpr int kFloats = kQ + kKV + kP;
  static constexpr int kBytes = kFloats * 4;
};

// Query rows per warp and warps per CTA of the fp32 tile kernel.
static const int kF32RowsPerWarp = tuning_knob("ATTN_F32_RW", 8) == 4 ? 4 : 8;
static const int kF32Warps = tuning_knob("ATTN_F32_WARPS", 8) == 4 ? 4 : 8;

// A lane's DL consecutive fp32 columns (DL = D/32: 2 at D=64, 4 at D=128) as
// one 8- or 16-byte access: the address is aligned to the access width.
template <int DL>
__device__ __forceinline__ void load_cols(const float* p, float (&v)[DL]) {
  static_assert(DL == 2 || DL == 4, "2 or 4 columns per lane");
  if constexpr (DL == 4) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  } else {
    const float2 x = *reinterpret_cast<const float2*>(p);
    v[0] = x.x; v[1] = x.y;
  }
}
template <int DL>
__device__ __forceinline__ void store_cols(float* p, const float* v, float scale) {
  if constexpr (DL == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0] * scale, v[1] * scale, v[2] * scale, v[3] * scale);
  } else {
    *reinterpret_cast<float2*>(p) = make_float2(v[0] * scale, v[1] * scale);
  }
}

template <int D, int RW, int W>
__global__ void __launch_bounds__(32 * W, W == 8 ? 2 : 1) attn_f32_kernel(const AttnArgs a) {
  DLI_PDL_ENTRY();
  using L = F32AttnSmem<D, RW, W>;
  constexpr int kThreads = L::kThreads;
  constexpr int DL = D / 32;  // output columns per lane
  constexpr int kRows = L::kRows;
  extern __shared__ __align__(16) float f32s[];
  float* sq = f32s;
  float* skv = f32s + L::kQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sp = skv + L::kKV + warp * kF32Keys * L::kPRow;  // this warp's P tile
  const int split = blockIdx.x, splits = gridDim.x;
  const int m0 = blockIdx.y * kRows;
  const int bh = blockIdx.z;
  const int h = bh % a.hq, b = bh / a.hq;
  const int kvh = h / a.group;
  const int kv_len = kv_len_of(a, b);
  const int off = kv_len - a.seq_q;
  const float* qbase = static_cast<const float*>(a.q) + b * a.q_sb + h * a.q_sh;
  const float* kbase = static_cast<const float*>(a.k) + b * a.k_sb + kvh * a.k_sh;
  const float* vbase = static_cast<const float*>(a.v) + b * a.k_sb + kvh * a.k_sh;

  // Q rows (zero past the sequence)
  for (int c = threadIdx.x; c < kRows * D / 4; c += kThreads) {
    const int r = c / (D / 4), d4 = (c % (D / 4)) * 4;
    const int qs = m0 + r;
    const float4 v = qs < a.seq_q ? *reinterpret_cast<const float4*>(qbase + static_cast<int64_t>(qs) * a.q_ss + d4)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(sq + r * L::kQRow + d4) = v;
  }
  int n_end = a.causal ? min(kv_len, m0 + kRows + off) : kv_len;
  n_end = max(n_end, 0);
  const int nblocks = (n_end + kF32Keys - 1) / kF32Keys;
  const int b0 = static_cast<int>(static_cast<int64_t>(split) * nblocks / splits);
  const int b1 = static_cast<int>(static_cast<int64_t>(split + 1) * nblocks / splits);

  auto load_block = [&](int blk, int stage) {
    float* kt = skv + stage * 2 * kF32Keys * L::kRow;
    float* vt = kt + kF32Keys * L::kRow;
    const uint32_t ks = static_cast<uint32_t>(__cvta_generic_to_shared(kt));
    const uint32_t vs = static_cast<uint32_t>(__cvta_generic_to_shared(vt));
    for (int c = threadIdx.x; c < kF32Keys * D / 4; c += kThreads) {
      const int r = c / (D / 4), d4 = (c % (D / 4)) * 4;
      const int key = blk * kF32Keys + r;
      const bool valid = key < n_end;
      const int64_t src = static_cast<int64_t>(valid ? key : 0) * D + d4;
      cp_async16(ks + (r * L::kRow + d4) * 4, kbase + src, valid);
      cp_async16(vs + (r * L::kRow + d4) * 4, vbase + src, valid);
    }
    cp_async_commit();
  };

  float o[RW][DL];
  float m_row[RW], l_row[RW];
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    m_row[i] = -INFINITY;
    l_row[i] = 0.f;
#pragma unroll
    for (int c = 0; c < DL; ++c) o[i][c] = 0.f;
  }
  const int r_base = warp * RW;
  const bool warp_rows = m0 + r_base < a.seq_q;  // the warp has at least one live row
  // last key the warp's last row may see (causal); blocks past it are skipped
  const int warp_key_end = m0 + r_base + RW + off;
  if (b0 < b1) load_block(b0, 0);
  for (int blk = b0; blk < b1; ++blk) {
    const int stage = (blk - b0) & 1;
    if (blk + 1 < b1) {
      load_block(blk + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* kt = skv + stage * 2 * kF32Keys * L::kRow;
    const float* vt = kt + kF32Keys * L::kRow;
    if (warp_rows && (!a.causal || blk * kF32Keys < warp_key_end)) {
      if constexpr (RW == 8) {
        // S for rows 2g, 2g+1 x keys c + 8j of the block
        const int g = lane >> 3, c = lane & 7;
        float sc[2][4];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int j = 0; j < 4; ++j) sc[t][j] = 0.f;
        const float* q0 = sq + (r_base + 2 * g) * L::kQRow;
#pragma unroll 4
        for (int d = 0; d < D; d += 4) {
          const float4 qa = *reinterpret_cast<const float4*>(q0 + d);
          const float4 qb = *reinterpret_cast<const float4*>(q0 + L::kQRow + d);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 kv = *reinterpret_cast<const float4*>(kt + (c + 8 * j) * L::kRow + d);
            sc[0][j] = fmaf(qa.x, kv.x, sc[0][j]);
            sc[0][j] = fmaf(qa.y, kv.y, sc[0][j]);
            sc[0][j] = fmaf(qa.z, kv.z, sc[0][j]);
            sc[0][j] = fmaf(qa.w, kv.w, sc[0][j]);
            sc[1][j] = fmaf(qb.x, kv.x, sc[1][j]);
            sc[1][j] = fmaf(qb.y, kv.y, sc[1][j]);
            sc[1][j] = fmaf(qb.z, kv.z, sc[1][j]);
            sc[1][j] = fmaf(qb.w, kv.w, sc[1][j]);
          }
        }
        // masked, scaled scores and each row's block maximum over its 8-lane group
        float gmax[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int qs = m0 + r_base + 2 * g + t;
          const int lim = a.causal ? min(kv_len, qs + off + 1) : kv_len;
          gmax[t] = -INFINITY;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int key = blk * kF32Keys + c + 8 * j;
            sc[t][j] = key < lim ? sc[t][j] * a.scale_log2 : -INFINITY;
            gmax[t] = fmaxf(gmax[t], sc[t][j]);
          }
#pragma unroll
          for (int x = 1; x < 8; x <<= 1) gmax[t] = fmaxf(gmax[t], __shfl_xor_sync(0xffffffffu, gmax[t], x));
        }
        // every lane: new maxima and rescale factors of all 8 rows
        float mown[2];
#pragma unroll
        for (int i = 0; i < RW; ++i) {
          const float bm = __shfl_sync(0xffffffffu, gmax[i & 1], (i >> 1) * 8);
          const float mnew = fmaxf(m_row[i], bm);
          const float alpha = mnew == -INFINITY ? 1.f : exp2f(m_row[i] - mnew);
          l_row[i] *= alpha;
          m_row[i] = mnew;
#pragma unroll
          for (int cc = 0; cc < DL; ++cc) o[i][cc] *= alpha;
        }
        // the lane's own rows' maxima (the same values as m_row[2g + t])
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          float mt = m_row[t];
#pragma unroll
          for (int gg = 1; gg < 4; ++gg) mt = g == gg ? m_row[2 * gg + t] : mt;
          mown[t] = mt;
        }
        // probabilities, written as [key][row] pairs, and each row's block sum
        float gsum[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p0 = mown[0] == -INFINITY ? 0.f : exp2f(sc[0][j] - mown[0]);
          const float p1 = mown[1] == -INFINITY ? 0.f : exp2f(sc[1][j] - mown[1]);
          gsum[0] += p0;
          gsum[1] += p1;
          *reinterpret_cast<float2*>(sp + (c + 8 * j) * L::kPRow + 2 * g) = make_float2(p0, p1);
        }
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int x = 1; x < 8; x <<= 1) gsum[t] += __shfl_xor_sync(0xffffffffu, gsum[t], x);
#pragma unroll
        for (int i = 0; i < RW; ++i) l_row[i] += __shfl_sync(0xffffffffu, gsum[i & 1], (i >> 1) * 8);
      } else {
        // scores of key (blk*32 + lane) for the warp's RW rows
        float sc[RW];
#pragma unroll
        for (int i = 0; i < RW; ++i) sc[i] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; d += 4) {
          const float4 kv = *reinterpret_cast<const float4*>(kt + lane * L::kRow + d);
#pragma unroll
          for (int i = 0; i < RW; ++i) {
            const float4 qv = *reinterpret_cast<const float4*>(sq + (r_base + i) * L::kQRow + d);
            sc[i] = fmaf(qv.x, kv.x, sc[i]);
            sc[i] = fmaf(qv.y, kv.y, sc[i]);
            sc[i] = fmaf(qv.z, kv.z, sc[i]);
            sc[i] = fmaf(qv.w, kv.w, sc[i]);
          }
        }
        const int key = blk * kF32Keys + lane;
        float pr[RW];
#pragma unroll
        for (int i = 0; i < RW; ++i) {
          const int qs = m0 + r_base + i;
          const int lim = a.causal ? min(kv_len, qs + off + 1) : kv_len;
          const float v = key < lim ? sc[i] * a.scale_log2 : -INFINITY;
          const float mnew = fmaxf(m_row[i], warp_max(v));
          const float alpha = mnew == -INFINITY ? 1.f : exp2f(m_row[i] - mnew);
          pr[i] = mnew == -INFINITY ? 0.f : exp2f(v - mnew);
          l_row[i] = l_row[i] * alpha + warp_sum(pr[i]);
          m_row[i] = mnew;
#pragma unroll
          for (int cc = 0; cc < DL; ++cc) o[i][cc] *= alpha;
        }
        // the lane's key row of P: [key][row], float4 stores
#pragma unroll
        for (int i = 0; i < RW; i += 4)
          *reinterpret_cast<float4*>(sp + lane * L::kPRow + i) = make_float4(pr[i], pr[i + 1], pr[i + 2], pr[i + 3]);
      }
      __syncwarp();
      // O += P V: lane owns columns lane*DL .. lane*DL+DL-1
#pragma unroll 4
      for (int j = 0; j < kF32Keys; ++j) {
        float vv[DL];
        load_cols<DL>(vt + j * L::kRow + lane * DL, vv);
#pragma unroll
        for (int i4 = 0; i4 < RW; i4 += 4) {
          const float4 p4 = *reinterpret_cast<const float4*>(sp + j * L::kPRow + i4);
          const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
          for (int ii = 0; ii < 4; ++ii)
#pragma unroll
            for (int c = 0; c < DL; ++c) o[i4 + ii][c] = fmaf(pj[ii], vv[c], o[i4 + ii][c]);
        }
      }
    }
    __syncthreads();  // the stage (and the P tile) is rewritten next iteration
  }

  auto store_row = [&](int r, const float* vals, float inv) {
    const int qs = m0 + r;
    if (qs >= a.seq_q) return;
    float* dst = static_cast<float*>(a.out) + b * a.o_sb + h * a.o_sh + static_cast<int64_t>(qs) * a.o_ss;
    store_cols<DL>(dst + lane * DL, vals, inv);
  };
  if (splits == 1) {
#pragma unroll
    for (int i = 0; i < RW; ++i) store_row(r_base + i, o[i], l_row[i] > 0.f ? 1.f / l_row[i] : 0.f);
    return;
  }
  // split-KV: publish (m, l, O) in the freed K/V stages (every warp passed the
  // loop's last __syncthreads and no cp.async is in flight) and merge across the
  // cluster in rank order
  float* st = skv;
  float* so = st;
  float* sm = st + kRows * D;
  float* sl = sm + kRows;
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    store_cols<DL>(so + (r_base + i) * D + lane * DL, o[i], 1.f);
    if (lane == 0) {
      sm[r_base + i] = m_row[i];
      sl[r_base + i] = l_row[i];
    }
  }
  cluster_sync();
  const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(st));
  const int rows_per = (kRows + splits - 1) / splits;
  for (int r = split * rows_per + warp; r < min(kRows, (split + 1) * rows_per); r += W) {
    float mm = -INFINITY;
    for (int s = 0; s < splits; ++s) {
      float v;
      asm volatile("ld.shared::cluster.f32 %0, [%1];"
                   : "=f"(v)
                   : "r"(mapa_shared(base + static_cast<uint32_t>((kRows * D + r) * 4), s))
                   : "memory");
      mm = fmaxf(mm, v);
    }
    float acc[DL], ll = 0.f;
#pragma unroll
    for (int c = 0; c < DL; ++c) acc[c] = 0.f;
    for (int s = 0; s < splits; ++s) {
      float ms, ls;
      asm volatile("ld.shared::cluster.f32 %0, [%1];"
                   : "=f"(ms)
                   : "r"(mapa_shared(base + static_cast<uint32_t>((kRows * D + r) * 4), s))
                   : "memory");
      asm volatile("ld.shared::cluster.f32 %0, [%1];"
                   : "=f"(ls)
                   : "r"(mapa_shared(base + static_cast<uint32_t>((kRows * D + kRows + r) * 4), s))
                   : "memory");
      const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - mm);
      ll += ls * w;
#pragma unroll
      for (int c = 0; c < DL; ++c) {  // scalar DSMEM loads: 4-byte aligned for any DL
        float x;
        asm volatile("ld.shared::cluster.f32 %0, [%1];"
                     : "=f"(x)
                     : "r"(mapa_shared(base + static_cast<uint32_t>((r * D + lane * DL + c) * 4), s))
                     : "memory");
        acc[c] += w * x;
      }
    }
    store_row(r, acc, ll > 0.f ? 1.f / ll : 0.f);
  }
  cluster_sync();  // every rank's shared memory stays alive until all reads are done
}

template <int D, int RW, int W>
dli_status launch_attn_f32_rw(const AttnArgs& args, cudaStream_t stream) {
  using L = F32AttnSmem<D, RW, W>;
  auto kern = attn_f32_kernel<D, RW, W>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kern), L::kBytes, "attention fp32");
  if (st != DLI_OK) return st;
  const int64_t tiles = ceil_div(args.seq_q, L::kRows);
  const int64_t rows = tiles * args.batch * args.hq;
  const int64_t blocks = ceil_div(args.seq_k, kF32Keys);
  // split the keys when the row tiles alone leave SMs idle (two CTAs per SM)
  int splits = static_cast<int>(std::min<int64_t>(8, std::max<int64_t>(1, ceil_div(2 * sm_count(), rows))));
  splits = static_cast<int>(std::min<int64_t>(splits, std::max<int64_t>(1, blocks / 2)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(tiles),
                     static_cast<unsigned>(static_cast<int64_t>(args.batch) * args.hq));
  cfg.blockDim = dim3(L::kThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (splits > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, kern, args);
  return check_launch("attention fp32");
}

template <int D>
dli_status launch_attn_f32(const AttnArgs& args, cudaStream_t stream) {
  if (kF32Warps == 8)
    return kF32RowsPerWarp == 4 ? launch_attn_f32_rw<D, 4, 8>(args, stream) : launch_attn_f32_rw<D, 8, 8>(args, stream);
  return kF32RowsPerWarp == 4 ? launch_attn_f32_rw<D, 4, 4>(args, stream) : launch_attn_f32_rw<D, 8, 4>(args, stream);
}

// ---- fp32 decode: few query rows per KV head ---------------------------------------
// CTA = (key split, KV head, sequence), 4 warps, each walking its own contiguous
// range of 32-key chunks for all R = seq_q * group (<= 8) query rows of the KV
// head at once: lane j scores key j from its own K row (D/4 independent 16-byte
// loads in flight) against the rows in shared memory, the online softmax runs
// per row across the warp, and for O += P V each lane owns D/32 columns of the
// key's V row (one coalesced 16-byte load per key). The four warps merge their
// (m, l, O) through shared memory, and the key splits of one (sequence, KV
// head) merge through distributed shared memory in rank order: exact fp32,
// deterministic, no workspace.
constexpr int kF32DecWarps = 4;

template <int D, int R>
__global__ void __launch_bounds__(128) attn_f32_decode_kernel(const AttnArgs a, int rows) {
  DLI_PDL_ENTRY();
  constexpr int DL = D / 32;
  __shared__ __align__(16) float sq[R][D];                  // query rows, pre-scaled by scale*log2(e)
  __shared__ __align__(16) float so[kF32DecWarps][R][D];    // per-warp O
  __shared__ float sm[kF32DecWarps][R], sl[kF32DecWarps][R];
  __shared__ __align__(16) float co[R][D];                  // this CTA's merged O (split merge source)
  __shared__ float cml[2][R];                               // its m and l
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, splits = gridDim.x;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int kv_len = kv_len_of(a, b);
  const int off = kv_len - a.seq_q;
  // row r = query position r / group, query head kvh * group + r % group
  for (int i = threadIdx.x; i < R * D; i += 128) {
    const int r = i / D, d = i - (i / D) * D;
    float v = 0.f;
    if (r < rows) {
      const int sqp = r / a.group, h = kvh * a.group + r % a.group;
      v = static_cast<const float*>(a.q)[b * a.q_sb + h * a.q_sh + static_cast<int64_t>(sqp) * a.q_ss + d] *
          a.scale_log2;
    }
    sq[r][d] = v;
  }
  __syncthreads();
  const float* kbase = static_cast<const float*>(a.k) + b * a.k_sb + kvh * a.k_sh;
  const float* vbase = static_cast<const float*>(a.v) + b * a.k_sb + kvh * a.k_sh;
  const int n_end = max(min(kv_len, a.seq_k), 0);  // never past the cache rows
  const int nchunks = (n_end + 31) / 32;
  const int c0 = static_cast<int>(static_cast<int64_t>(split) * nchunks / splits);
  const int c1 = static_cast<int>(static_cast<int64_t>(split + 1) * nchunks / splits);
  const int w0 = c0 + (c1 - c0) * warp / kF32DecWarps, w1 = c0 + (c1 - c0) * (warp + 1) / kF32DecWarps;
  int lim[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int sqp = r / a.group;
    lim[r] = r < rows ? min(a.causal ? min(kv_len, sqp + off + 1) : kv_len, n_end) : 0;
  }
  float m[R], l[R], o[R][DL];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int c = 0; c < DL; ++c) o[r][c] = 0.f;
  }
  for (int ch = w0; ch < w1; ++ch) {
    const int key = ch * 32 + lane;
    const float* kr = kbase + static_cast<int64_t>(key < n_end ? key : 0) * D;
    float sc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) sc[r] = 0.f;
#pragma unroll 8
    for (int d = 0; d < D; d += 4) {
      const float4 kv = __ldg(reinterpret_cast<const float4*>(kr + d));
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float4 qv = *reinterpret_cast<const float4*>(&sq[r][d]);
        sc[r] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, sc[r]))));
      }
    }
    float pr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float v = key < lim[r] ? sc[r] : -INFINITY;
      const float mnew = fmaxf(m[r], warp_max(v));
      const float alpha = mnew == -INFINITY ? 1.f : exp2f(m[r] - mnew);
      pr[r] = mnew == -INFINITY ? 0.f : exp2f(v - mnew);
      l[r] = l[r] * alpha + warp_sum(pr[r]);
      m[r] = mnew;
#pragma unroll
      for (int c = 0; c < DL; ++c) o[r][c] *= alpha;
    }
    const int nk = min(32, n_end - ch * 32);
    auto load_v = [&](int j, float (&vv)[DL]) {
      const float* vr = vbase + static_cast<int64_t>(ch * 32 + j) * D + lane * DL;
      if constexpr (DL == 4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(vr));
        vv[0] = x.x; vv[1] = x.y; vv[2] = x.z; vv[3] = x.w;
      } else {
        const float2 x = __ldg(reinterpret_cast<const float2*>(vr));
        vv[0] = x.x; vv[1] = x.y;
      }
    };
    auto add_pv = [&](int j, const float (&vv)[DL]) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float pj = __shfl_sync(0xffffffffu, pr[r], j);
#pragma unroll
        for (int c = 0; c < DL; ++c) o[r][c] = fmaf(pj, vv[c], o[r][c]);
      }
    };
    if (nk == 32) {
      // a full chunk: 8 V rows in flight per lane before they are used (a loop
      // of one load per key keeps too few bytes in flight to reach HBM rate);
      // the FMA order per output is the same as the loop below
      for (int j0 = 0; j0 < 32; j0 += 8) {
        float vv[8][DL];
#pragma unroll
        for (int u = 0; u < 8; ++u) load_v(j0 + u, vv[u]);
#pragma unroll
        for (int u = 0; u < 8; ++u) add_pv(j0 + u, vv[u]);
      }
    } else {
      for (int j = 0; j < nk; ++j) {
        float vv[DL];
        load_v(j, vv);
        add_pv(j, vv);
      }
    }
  }
  // merge the four warps (in warp order) into this CTA's (m, l, O)
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int c = 0; c < DL; ++c) so[warp][r][lane * DL + c] = o[r][c];
    if (lane == 0) {
      sm[warp][r] = m[r];
      sl[warp][r] = l[r];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * D; i += 128) {
    const int r = i / D, d = i - (i / D) * D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kF32DecWarps; ++w) mm = fmaxf(mm, sm[w][r]);
    float acc = 0.f, ll = 0.f;
#pragma unroll
    for (int w = 0; w < kF32DecWarps; ++w) {
      const float wt = sm[w][r] == -INFINITY ? 0.f : exp2f(sm[w][r] - mm);
      acc += so[w][r][d] * wt;
      ll += sl[w][r] * wt;
    }
    co[r][d] = acc;
    if (d == 0) {
      cml[0][r] = mm;
      cml[1][r] = ll;
    }
  }
  auto store = [&](int r, int d, float val) {
    if (r >= rows) return;
    const int sqp = r / a.group, h = kvh * a.group + r % a.group;
    static_cast<float*>(a.out)[b * a.o_sb + h * a.o_sh + static_cast<int64_t>(sqp) * a.o_ss + d] = val;
  };
  if (splits == 1) {
    __syncthreads();
    for (int i = threadIdx.x; i < R * D; i += 128) {
      const int r = i / D, d = i - (i / D) * D;
      store(r, d, cml[1][r] > 0.f ? co[r][d] / cml[1][r] : 0.f);
    }
    return;
  }
  // split-KV: merge the cluster's ranks in rank order; rank s writes elements s, s + S, ...
  cluster_sync();
  const uint32_t co_l = static_cast<uint32_t>(__cvta_generic_to_shared(&co[0][0]));
  const uint32_t ml_l = static_cast<uint32_t>(__cvta_generic_to_shared(&cml[0][0]));
  for (int i = split * 128 + threadIdx.x; i < R * D; i += splits * 128) {
    const int r = i / D, d = i - (i / D) * D;
    float ms[8], ls[8], os[8];
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) {
      if (s2 < splits) {
        asm volatile("ld.shared::cluster.f32 %0, [%1];"
                     : "=f"(ms[s2]) : "r"(mapa_shared(ml_l + r * 4, s2)) : "memory");
        asm volatile("ld.shared::cluster.f32 %0, [%1];"
                     : "=f"(ls[s2]) : "r"(mapa_shared(ml_l + (R + r) * 4, s2)) : "memory");
        asm volatile("ld.shared::cluster.f32 %0, [%1];"
                     : "=f"(os[s2]) : "r"(mapa_shared(co_l + (r * D + d) * 4, s2)) : "memory");
      }
    }
    float mm = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2)
      if (s2 < splits) mm = fmaxf(mm, ms[s2]);
    float acc = 0.f, ll = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) {
      if (s2 < splits) {
        const float wt = ms[s2] == -INFINITY ? 0.f : exp2f(ms[s2] - mm);
        acc += os[s2] * wt;
        ll += ls[s2] * wt;
      }
    }
    store(r, d, ll > 0.f ? acc / ll : 0.f);
  }
  cluster_sync();  // every rank's shared memory stays alive until all reads are done
}

template <int D, int R>
dli_status launch_attn_f32_decode(const AttnArgs& args, int rows, cudaStream_t stream) {
  const int64_t heads = static_cast<int64_t>(args.batch) * args.hkv;
  const int64_t keys = args.seq_k;  // the cache rows (or the dense key count) bound every sequence
  const int64_t nchunks = ceil_div(std::max<int64_t>(keys, 1), 32);
  // enough CTAs for four per SM, each warp keeping >= 2 chunks of 32 keys
  int splits = static_cast<int>(std::min<int64_t>(8, std::max<int64_t>(1, ceil_div(4 * sm_count(), heads))));
  splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(splits, nchunks / (2 * kF32DecWarps))));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(args.hkv), static_cast<unsigned>(args.batch));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (splits > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, attn_f32_decode_kernel<D, R>, args, rows);
  return check_launch("attention fp32 decode");
}

// The fp32 decode kernel serves <= 8 query rows per KV head, head_dim 64/128,
// 16-byte aligned K/V rows (DLI_SM100_ATTN_F32_DECODE=0 sends them to the tile kernel).
bool f32_decode_ok(const AttnArgs& a) {
  static const bool on = tuning_knob("ATTN_F32_DECODE", 1) != 0;
  const int64_t rows = static_cast<int64_t>(a.seq_q) * a.group;
  if (!on || rows < 1 || rows > 8 || (a.head_dim != 64 && a.head_dim != 128)) return false;
  if (a.batch > 65535 || a.hkv > 65535 || !aligned(a.k, 16) || !aligned(a.v, 16)) return false;
  return a.k_sb % 4 == 0 && a.k_sh % 4 == 0;
}

dli_status run_attn_f32_decode(const AttnArgs& a, cudaStream_t stream) {
  const int rows = a.seq_q * a.group;
  const int r = rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8;
  if (a.head_dim == 64) {
    switch (r) {
      case 1: return launch_attn_f32_decode<64, 1>(a, rows, stream);
      case 2: return launch_attn_f32_decode<64, 2>(a, rows, stream);
      case 4: return launch_attn_f32_decode<64, 4>(a, rows, stream);
      default: return launch_attn_f32_decode<64, 8>(a, rows, stream);
    }
  }
  switch (r) {
    case 1: return launch_attn_f32_decode<128, 1>(a, rows, stream);
    case 2: return launch_attn_f32_decode<128, 2>(a, rows, stream);
    case 4: return launch_attn_f32_decode<128, 4>(a, rows, stream);
    default: return launch_attn_f32_decode<128, 8>(a, rows, stream);
  }
}

bool f32_attention_ok(const AttnArgs& a) {
  static const bool on = tuning_knob("ATTN_F32", 1) != 0;
  if (!on || (a.head_dim != 64 && a.head_dim != 128)) return false;
  if (static_cast<int64_t>(a.batch) * a.hq > 65535 || ceil_div(a.seq_q, 4 * kF32RowsPerWarp) > 65535) return false;
  for (const void* ptr : {a.q, a.k, a.v, static_cast<const void*>(a.out)})
    if (!aligned(ptr, 16)) return false;
  for (int64_t s : {a.q_sb, a.q_sh, a.q_ss, a.o_sb, a.o_sh, a.o_ss, a.k_sb, a.k_sh})
    if (s % 4 != 0) return false;
  return true;
}

// ---- host dispatch ----------------------------------------------------------------------
struct DecodePlan {
  bool decode = false;
  bool cluster = false;  // attn_decode_cluster_kernel (<= 8 query rows per KV head)
  int splits = 1;
  size_t workspace = 0;
};

// K/V stages of the cluster decode kernel: 3 (two CTAs per SM at D = 128) or 2.
static const int kClusterStages = tuning_knob("ATTN_CLUSTER_STAGES", 3) == 2 ? 2 : 3;

// DLI_SM100_ATTN_DECODE_TMA: 1 K/V blocks of the cluster decode kernel by TMA
// with mbarrier stages; 0 (default) by cp.async with a CTA barrier per block.
// Measured at the Qwen2-7B decode shape (B 32, context 2304): 31.2 us by TMA
// against 30.2 us by cp.async, so the barrier per block is not what bounds it.
static const bool kDecodeTma = tuning_knob("ATTN_DECODE_TMA", 0) != 0;

template <int D, int STAGES>
int cluster_decode_occupancy(int cluster) {
  using L = DecodeClusterSmem<__nv_bfloat16, D, STAGES, true>;  // the larger of the two layouts
  auto kern = attn_decode_cluster_kernel<__nv_bfloat16, D, STAGES, true>;
  if (ensure_smem(reinterpret_cast<const void*>(kern), L::kBytes, "attention decode") != DLI_OK) return 0;
  int n = 0;
  if (cluster <= 1) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 128, L::kBytes) != cudaSuccess) n = 0;
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(cluster), 1, 1);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = L::kBytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(cluster);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  return n;
}

// CTAs per SM (cluster <= 1) or resident clusters, cached per device.
int cluster_decode_capacity(int head_dim, int cluster) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const auto key = std::make_tuple(dev, head_dim, kClusterStages, cluster);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (head_dim == 64)
    n = kClusterStages == 3 ? cluster_decode_occupancy<64, 3>(cluster) : cluster_decode_occupancy<64, 2>(cluster);
  else
    n = kClusterStages == 3 ? cluster_decode_occupancy<128, 3>(cluster) : cluster_decode_occupancy<128, 2>(cluster);
  cache[key] = n;
  return n;
}

DecodePlan plan_decode(int64_t batch, int64_t hkv, int64_t group, int64_t seq_q, int64_t max_kv,
                       int64_t head_dim) {
  DecodePlan p;
  if (group * seq_q > 16) return p;
  p.decode = true;
  const int64_t pairs = batch * hkv;
  const int64_t blocks = std::max<int64_t>(1, ceil_div(max_kv, 64));
  static const bool kClusterOn = tuning_knob("ATTN_CLUSTER", 1) != 0;
  if (group * seq_q <= 8 && kClusterOn) {
    // One resident wave: the largest cluster size S <= 8 with pairs * S CTAs all
    // resident at once and every split holding >= 1 key block.
    p.cluster = true;
    const int64_t slots = static_cast<int64_t>(std::max(1, cluster_decode_capacity(static_cast<int>(head_dim), 1))) *
                          sm_count();
    for (int s = 8; s >= 2; --s) {
      if (pairs * s <= slots && s <= blocks && pairs <= cluster_decode_capacity(static_cast<int>(head_dim), s)) {
        p.splits = s;
        break;
      }
    }
    return p;
  }
  // Few, long splits measure best: each split pays a pipeline fill, a 4-warp
  // merge and a partial round trip, so splits only need to fill the SMs once.
  static const int kWaves = tuning_knob("ATTN_WAVES", 1);
  static const int kMinBlocks = std::max(1, tuning_knob("ATTN_MIN_BLOCKS", 1));
  const int64_t target = static_cast<int64_t>(kWaves) * (kDecodeStages == 2 ? 3 : 2) * sm_count();
  // as many splits as keep every CTA resident at once: a partial second wave
  // costs nearly a whole CTA lifetime (measured 59 us -> 41 us at the 7B shape)
  int64_t splits = std::max<int64_t>(1, target / pairs);
  splits = std::min<int64_t>(splits, std::max<int64_t>(1, blocks / kMinBlocks));
  splits = std::min<int64_t>(splits, kMaxSplits);
  p.splits = static_cast<int>(splits);
  if (p.splits > 1)
    p.workspace = static_cast<size_t>(pairs * p.splits) * (16 * head_dim + 32) * sizeof(float);
  return p;
}

bool tc_head_dim(int64_t d) { return d == 64 || d == 128; }

template <typename T, int D, int STAGES>
dli_status launch_decode(const AttnArgs& args, const DecodePlan& plan, cudaStream_t stream) {
  constexpr int kSmem = 2 * STAGES * 64 * D * 2 + 16 * D * 4 + 128 * 4;
  auto kern = attn_decode_kernel<T, D, STAGES>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kern), kSmem, "attention decode");
  if (st != DLI_OK) return st;
  dim3 grid(plan.splits, args.hkv, args.batch);
  launch_pdl(kern, grid, dim3(128), kSmem, stream, args);
  return DLI_OK;
}

// The K/V tensor maps of the TMA decode kernel: 4-D [batch, Hkv, cache rows, D]
// with 64-key x 64-element boxes. False (and the cp.async kernel serves the
// call) when the layout is outside what a map can describe.
template <int D>
bool decode_kv_maps(const AttnArgs& a, bool bf16, CUtensorMap* tk, CUtensorMap* tv) {
  if (a.k_sh % D != 0 || a.k_sh % 8 != 0 || a.k_sb % 8 != 0 || a.k_sb < a.k_sh) return false;
  const int64_t rows = a.k_sh / D;
  if (rows < 1 || rows > (1ll << 30)) return false;
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(rows), static_cast<uint64_t>(a.hkv),
                            static_cast<uint64_t>(a.batch)};
  const uint64_t strides[3] = {static_cast<uint64_t>(D * 2), static_cast<uint64_t>(a.k_sh * 2),
                               static_cast<uint64_t>(a.k_sb * 2)};
  const uint32_t box[4] = {64u, 64u, 1u, 1u};
  if (make_map_4d(tk, a.k, bf16, dims, strides, box) != DLI_OK) return false;
  if (make_map_4d(tv, a.v, bf16, dims, strides, box) != DLI_OK) return false;
  return true;
}

template <typename T, int D, int STAGES>
dli_status launch_decode_cluster(const AttnArgs& args, const DecodePlan& plan, cudaStream_t stream) {
  CUtensorMap tk, tv;
  const bool tma = kDecodeTma && decode_kv_maps<D>(args, std::is_same<T, __nv_bfloat16>::value, &tk, &tv);
  if (!tma) {
    std::memset(&tk, 0, sizeof(tk));
    std::memset(&tv, 0, sizeof(tv));
  }
  const unsigned smem =
      tma ? DecodeClusterSmem<T, D, STAGES, true>::kBytes : DecodeClusterSmem<T, D, STAGES, false>::kBytes;
  auto kern = tma ? attn_decode_cluster_kernel<T, D, STAGES, true> : attn_decode_cluster_kernel<T, D, STAGES, false>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kern), smem, "attention decode");
  if (st != DLI_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(plan.splits), static_cast<unsigned>(args.hkv),
                     static_cast<unsigned>(args.batch));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (plan.splits > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(plan.splits);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, kern, args, tk, tv);
  return check_launch("attention decode");
}

template <typename T, int D>
dli_status launch_tc_attention(const AttnArgs& args, const DecodePlan& plan, cudaStream_t stream) {
  if (plan.decode && plan.cluster) {
    return kClusterStages == 3 ? launch_decode_cluster<T, D, 3>(args, plan, stream)
                               : launch_decode_cluster<T, D, 2>(args, plan, stream);
  }
  if (plan.decode) {
    const dli_status st = kDecodeStages == 3 ? launch_decode<T, D, 3>(args, plan, stream)
                                             : launch_decode<T, D, 2>(args, plan, stream);
    if (st != DLI_OK) return st;
    if (plan.splits > 1) {
      dim3 cg(args.hkv, args.batch);
      launch_pdl(attn_combine_kernel<T>, cg, dim3(256), 0, stream, args);
    }
    return check_launch("attention decode", plan.splits > 1 ? 2 : 1);
  }
  constexpr int kSmem = (64 * D + 4 * 64 * D) * 2;
  auto kern = attn_prefill_kernel<T, D>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kern), kSmem, "attention prefill");
  if (st != DLI_OK) return st;
  dim3 grid(static_cast<unsigned>(ceil_div(args.seq_q, 64)), args.hq, args.batch);
  launch_pdl(kern, grid, dim3(128), kSmem, stream, args);
  return check_launch("attention prefill");
}

dli_status run_attention(AttnArgs& args, dli_dtype dtype, int64_t max_kv, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream) {
  const bool tc = (dtype == DLI_DTYPE_BF16 || dtype == DLI_DTYPE_F16) &&
                  tc_head_dim(args.head_dim) && aligned(args.q, 16) && aligned(args.k, 16) &&
                  aligned(args.v, 16) && aligned(args.out, 4);
  if (tc) {
    const DecodePlan plan = plan_decode(args.batch, args.hkv, args.group, args.seq_q, max_kv, args.head_dim);
    if (!plan.decode) {
      // prefill: the tcgen05 kernel (TMEM accumulators, TMA K/V) when the layout allows
      FmhaArgs f{};
      f.q = args.q;
      f.k = args.k;
      f.v = args.v;
      f.out = args.out;
      f.q_sb = args.q_sb;
      f.q_sh = args.q_sh;
      f.q_ss = args.q_ss;
      f.o_sb = args.o_sb;
      f.o_sh = args.o_sh;
      f.o_ss = args.o_ss;
      f.k_sb = args.k_sb;
      f.k_sh = args.k_sh;
      f.batch = args.batch;
      f.hq = args.hq;
      f.hkv = args.hkv;
      f.seq_q = args.seq_q;
      f.dense_kv = args.seq_k;
      f.head_dim = args.head_dim;
      f.positions = args.positions;
      f.scale_log2 = args.scale_log2;
      f.causal = args.causal;
      if (fmha_supported(f, dtype)) {
        const dli_status st = run_fmha_prefill(f, dtype, stream);
        if (st != DLI_ERR_UNSUPPORTED) return st;
      }
      if (fmha_required())
        return fail(DLI_ERR_UNSUPPORTED, "attention: the tcgen05 prefill kernel cannot serve this layout "
                                         "(DLI_SM100_ATTN_FMHA=2)");
    }
    if (plan.decode && !plan.cluster && plan.splits > 1) {
      if (workspace == nullptr || workspace_bytes < plan.workspace)
        return fail(DLI_ERR_WORKSPACE, "attention: workspace too small (need " +
                                           std::to_string(plan.workspace) + " bytes)");
      args.part_o = static_cast<float*>(workspace);
      args.part_ml = args.part_o + static_cast<int64_t>(args.batch) * args.hkv * plan.splits * 16 * args.head_dim;
    }
    args.splits = plan.splits;
    args.err = device_error_word();
    if (dtype == DLI_DTYPE_BF16)
      return args.head_dim == 64 ? launch_tc_attention<__nv_bfloat16, 64>(args, plan, stream)
                                 : launch_tc_attention<__nv_bfloat16, 128>(args, plan, stream);
    return args.head_dim == 64 ? launch_tc_attention<__half, 64>(args, plan, stream)
                               : launch_tc_attention<__half, 128>(args, plan, stream);
  }
  if (dtype == DLI_DTYPE_F32 && f32_decode_ok(args)) return run_attn_f32_decode(args, stream);
  if (dtype == DLI_DTYPE_F32 && f32_attention_ok(args))
    return args.head_dim == 64 ? launch_attn_f32<64>(args, stream) : launch_attn_f32<128>(args, stream);
  if (args.head_dim > 256) return fail(DLI_ERR_UNSUPPORTED, "attention: head_dim > 256");
  const int64_t rows = static_cast<int64_t>(args.batch) * args.hq * args.seq_q;
  const int warps = 4;
  const unsigned grid = static_cast<unsigned>(ceil_div(rows, warps));
  const size_t smem = warps * args.head_dim * sizeof(float);
  const dli_status st = dispatch_float(dtype, "attention", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(attn_fallback_kernel<T>, dim3(grid), dim3(warps * 32), smem, stream, args);
  });
  if (st != DLI_OK) return st;
  return check_launch("attention fallback");
}

size_t attention_ws(int64_t batch, int64_t hq, int64_t hkv, int64_t seq_q, int64_t max_kv,
                    int64_t head_dim, dli_dtype dtype) {
  if (batch <= 0 || hq <= 0 || hkv <= 0 || hq % hkv != 0) return 0;
  const bool tc = (dtype == DLI_DTYPE_BF16 || dtype == DLI_DTYPE_F16) && tc_head_dim(head_dim);
  if (!tc) return 0;
  const DecodePlan plan = plan_decode(batch, hkv, hq / hkv, seq_q, max_kv, head_dim);
  return plan.decode ? plan.workspace : 0;
}

}  // namespace
}  // namespace dli_sm100

using namespace dli_sm100;

extern "C" size_t dli_sm100_attention_workspace_size(int64_t batch, int64_t q_heads,
                                                     int64_t kv_heads, int64_t seq_q,
                                                     int64_t seq_k, int64_t head_dim,
                                                     dli_dtype dtype) {
  return attention_ws(batch, q_heads, kv_heads, seq_q, seq_k, head_dim, dtype);
}

extern "C" dli_status dli_sm100_attention(const void* q, const void* k, const void* v, void* out,
                                          int64_t batch, int64_t q_heads, int64_t kv_heads,
                                          int64_t seq_q, int64_t seq_k, int64_t kv_capacity,
                                          int64_t head_dim, int causal, float scale,
                                          dli_dtype dtype, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || seq_q < 0 || seq_k < 0 || head_dim <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "attention: bad sizes");
  if (q_heads % kv_heads != 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "attention: q heads must be a multiple of kv heads");
  if (kv_capacity < seq_k) return fail(DLI_ERR_INVALID_ARGUMENT, "attention: kv_capacity < seq_k");
  if (!is_float_dtype(dtype)) return fail(DLI_ERR_INVALID_ARGUMENT, "attention expects a float dtype");
  if (batch == 0 || seq_q == 0) return ok();
  if (seq_k == 0) return fail(DLI_ERR_INVALID_ARGUMENT, "attention: no keys");
  if (seq_q > (1 << 30) || seq_k > (1 << 30)) return fail(DLI_ERR_UNSUPPORTED, "attention: sequence too long");
  AttnArgs args{};
  args.q = q;
  args.k = k;
  args.v = v;
  args.out = out;
  args.q_sb = q_heads * seq_q * head_dim;
  args.q_sh = seq_q * head_dim;
  args.q_ss = head_dim;
  args.o_sb = args.q_sb;
  args.o_sh = args.q_sh;
  args.o_ss = args.q_ss;
  args.k_sb = kv_heads * kv_capacity * head_dim;
  args.k_sh = kv_capacity * head_dim;
  args.batch = static_cast<int>(batch);
  args.hq = static_cast<int>(q_heads);
  args.hkv = static_cast<int>(kv_heads);
  args.group = static_cast<int>(q_heads / kv_heads);
  args.seq_q = static_cast<int>(seq_q);
  args.seq_k = static_cast<int>(seq_k);
  args.head_dim = static_cast<int>(head_dim);
  args.positions = nullptr;
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  args.scale_log2 = sc * kLog2e;
  args.causal = causal ? 1 : 0;
  return run_attention(args, dtype, seq_k, workspace, workspace_bytes, as_stream(stream));
}

extern "C" size_t dli_sm100_attention_kvcache_workspace_size(int64_t batch, int64_t seq,
                                                             int64_t q_heads, int64_t kv_heads,
                                                             int64_t capacity, int64_t head_dim,
                                                             dli_dtype dtype) {
  return attention_ws(batch, q_heads, kv_heads, seq, capacity, head_dim, dtype);
}

extern "C" dli_status dli_sm100_attention_kvcache(const void* q, const void* cache_k,
                                                  const void* cache_v, const int64_t* positions,
                                                  void* out, int64_t batch, int64_t seq,
                                                  int64_t q_heads, int64_t kv_heads,
                                                  int64_t capacity, int64_t head_dim, float scale,
                                                  dli_dtype dtype, void* workspace,
                                                  size_t workspace_bytes, void* stream) {
  if (batch < 0 || seq < 0 || q_heads <= 0 || kv_heads <= 0 || capacity <= 0 || head_dim <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "attention_kvcache: bad sizes");
  if (q_heads % kv_heads != 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "attention_kvcache: q heads must be a multiple of kv heads");
  if (positions == nullptr) return fail(DLI_ERR_INVALID_ARGUMENT, "attention_kvcache: positions required");
  if (!is_float_dtype(dtype)) return fail(DLI_ERR_INVALID_ARGUMENT, "attention_kvcache expects a float dtype");
  if (batch == 0 || seq == 0) return ok();
  AttnArgs args{};
  args.q = q;
  args.k = cache_k;
  args.v = cache_v;
  args.out = out;
  args.q_sb = seq * q_heads * head_dim;
  args.q_sh = head_dim;
  args.q_ss = q_heads * head_dim;
  args.o_sb = args.q_sb;
  args.o_sh = args.q_sh;
  args.o_ss = args.q_ss;
  args.k_sb = kv_heads * capacity * head_dim;
  args.k_sh = capacity * head_dim;
  args.batch = static_cast<int>(batch);
  args.hq = static_cast<int>(q_heads);
  args.hkv = static_cast<int>(kv_heads);
  args.group = static_cast<int>(q_heads / kv_heads);
  args.seq_q = static_cast<int>(seq);
  args.seq_k = static_cast<int>(capacity);
  args.head_dim = static_cast<int>(head_dim);
  args.positions = positions;
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  args.scale_log2 = sc * kLog2e;
  args.causal = 1;
  return run_attention(args, dtype, capacity, workspace, workspace_bytes, as_stream(stream));
}

// ---- attention over a KV cache without any allocation --------------------------------
// Some callers cannot allocate device memory at all: code running inside a
// memory budget fixed up front (a serving loop that must not grow its
// footprint), hosts whose allocator is owned by another runtime, or callers that
// must not take the allocator's locks on their hot path. For them this variant
// takes the split-KV partials (the only scratch the decode path needs) from a
// file-scope device array of fixed size instead of a caller workspace.
namespace dli_sm100 {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB, held by every GPU that loads the library
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_noalloc_scratch on the current device. In host code the
// array's name is only a stand-in for the symbol, so the address is resolved
// once per device with that device current (cudaGetSymbolAddress) and cached.
dli_status noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(DLI_ERR_CUDA, std::string("no-alloc scratch: ") + cudaGetErrorString(err));
  if (dev < 0 || dev >= 64) return fail(DLI_ERR_UNSUPPORTED, "no-alloc scratch: device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr)
      return fail(DLI_ERR_CUDA, std::string("no-alloc scratch address: ") + cudaGetErrorString(err));
    addr[dev] = p;
  }
  *out = addr[dev];
  return DLI_OK;
}

}  // namespace
}  // namespace dli_sm100

extern "C" size_t dli_sm100_attention_kvcache_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

extern "C" dli_status dli_sm100_attention_kvcache_noalloc(const void* q, const void* cache_k,
                                                          const void* cache_v, const int64_t* positions,
                                                          void* out, int64_t batch, int64_t seq,
                                                          int64_t q_heads, int64_t kv_heads,
                                                          int64_t capacity, int64_t head_dim, float scale,
                                                          dli_dtype dtype, void* stream) {
  if (batch < 0 || seq < 0 || q_heads <= 0 || kv_heads <= 0 || capacity <= 0 || head_dim <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "attention_kvcache_noalloc: bad sizes");
  if (q_heads % kv_heads != 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "attention_kvcache_noalloc: q heads must be a multiple of kv heads");
  const size_t need = attention_ws(batch, q_heads, kv_heads, seq, capacity, head_dim, dtype);
  if (need > kNoAllocScratchBytes)
    return fail(DLI_ERR_WORKSPACE, "attention_kvcache_noalloc: this shape needs " + std::to_string(need) +
                                       " bytes of scratch, more than the fixed " +
                                       std::to_string(kNoAllocScratchBytes) +
                                       "; use dli_sm100_attention_kvcache with a caller workspace");
  void* scratch = nullptr;
  if (need > 0) {
    const dli_status st = noalloc_scratch(&scratch);
    if (st != DLI_OK) return st;
  }
  // The partials need no initial value: every split slot the merge reads is written
  // by the same call first, so leftover contents of an earlier call are harmless.
  return dli_sm100_attention_kvcache(q, cache_k, cache_v, positions, out, batch, seq, q_heads, kv_heads,
                                     capacity, head_dim, scale, dtype, scratch, need, stream);
}
