// Prefill attention on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Semantics are those of the reference attention operator
// (python/dli_ops/aot/attention/kernel.py:5-62): softmax(q k^T * scale) v with
// the bottom-right causal mask (query row i of Sq sees key j iff
// j <= i + Sk - Sq, kernel.py:35,49-50); GQA query head h reads KV head
// h / (Hq / Hkv).
//
// One CTA = 128 query rows of one (sequence, query head); 192 threads:
//   warp 0     TMA producer: the Q tile once, then 128-key K and V blocks
//              (4-D tensor maps over the strided q and the [B, Hkv, rows, D]
//              K/V layout, 128-byte swizzle) into a 3-deep K ring and a 2/3-deep
//              V ring, in the order the MMA warp consumes them;
//   warp 1     TMEM allocator (all 512 columns) and single-thread MMA issuer:
//                S_j = Q K_j^T   (M 128, N 128, K D; both operands K-major)
//                O  += P_j V_j   (M 128, N D, K 128; V is the MN-major B operand)
//              into S buffers at TMEM columns 0/128 and O at column 256, in the
//              order S_0, S_1, O+=P_0V_0, S_2, O+=P_1V_1, ... so the next S is
//              on the tensor pipe while the softmax warps work on the current one;
//   warps 2-5  softmax, one thread per query row (its TMEM lane): read the S row
//              (tcgen05.ld), mask, online max/sum in fp32, write P = exp2(S*scale
//              - m) as bf16/f16 (the A operand of O += P V) back over the first
//              half of the same S buffer with tcgen05.st (or, with the P-in-shared
//              variant, into a 128-byte-swizzled shared tile), and at the end
//              read O, divide by the row sum, write it over the Q tile in
//              shared memory and store the tile with TMA.
// The running maximum is only moved when a block raises it by more than 8
// (log2 units): until then P values up to 2^8 are accumulated against the old
// maximum, which is exact in fp32 and in the bf16/f16 range, so O in TMEM is
// rescaled (tcgen05.ld / st by the owning warp, after the previous P V has
// completed) only a few times per row instead of once per block.
//
// Synchronisation (all mbarriers, every wait bounded; a timeout sets the device
// error word and winds the CTA down): q_full; k_full/k_empty and v_full/v_empty
// per ring stage; s_full (MMA commit) and s_empty (4 softmax warps) per S
// buffer; p_full (4 softmax warps) per P; o_done (MMA commit after each P V):
// the softmax warps wait for it before they rescale O (and, with P in shared
// memory, before they rewrite the single P tile). A P in tensor memory needs
// no such wait: P_j sits in S_j's buffer, and S_{j+2}, the next write there,
// is issued after P_j V_j, which the tensor pipe executes first. A rescale at
// block j may wait on o_done's parity because S_j's commit already covered
// P V_{j-2}, so o_done is at most one phase behind; before the final read of
// O it may be two behind, so that read waits on mma_done, committed once after
// the last MMA.
//
// Keys at or past a sequence's length are masked; V rows past the length that
// exist in memory (stale cache rows) are zeroed in shared memory before the
// last P V, so a stale non-finite value cannot reach O through a zero weight.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "fmha.cuh"
#include "tcgen05.cuh"

namespace dli_sm100 {
namespace {

constexpr int kFmhaThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P <= 2^8 before O is rescaled

// Shared-memory and tensor-memory plan per head dim and key-block width. Keys
// per block 128: one CTA per SM (230 KB, all 512 TMEM columns). Keys per block
// 64: two CTAs per SM (<= 113 KB and 256 TMEM columns each), so one CTA's
// prologue, epilogue and softmax latency overlap the other's MMAs.
// PT: P goes to tensor memory over the S buffer it was computed from (the A
// operand of O += P V read from TMEM), which frees the shared P tile for a
// third K stage (64-key blocks) or V stage (128-key blocks).
template <int D, int BN_, bool PT>
struct FmhaLayout {
  static constexpr int BM = 128;  // query rows per CTA (tcgen05 M)
  static constexpr int BN = BN_;  // keys per block
  static constexpr int kCtasPerSm = BN_ == 64 ? 2 : 1;
  static constexpr int KST = BN_ == 128 ? 3 : ((D == 128 && !PT) ? 2 : 3);
  static constexpr int VST = BN_ == 128 ? ((D == 128 && !PT) ? 2 : 3) : 2;
  static constexpr int kBox = 128 * 128;                   // one 128-row x 64-element box
  static constexpr int kQBytes = (D / 64) * kBox;
  static constexpr int kKVBytes = (D / 64) * BN * 128;     // one K or V block
  static constexpr int kPBytes = PT ? 0 : (BN / 64) * kBox;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + KST * kKVBytes;
  static constexpr int kPOff = kVOff + VST * kKVBytes;
  static constexpr int kBarOff = kPOff + kPBytes;
  // q_full, k_full[KST], k_empty[KST], v_full[VST], v_empty[VST], s_full[2],
  // s_empty[2], p_full, o_done, mma_done
  static constexpr int kBars = 1 + 2 * KST + 2 * VST + 4 + 3;
  // One CTA per SM rounds its base up to 1 KiB inside the allocation; two CTAs
  // per SM have no room for that slack and rely on the dynamic shared memory
  // base being 1 KiB aligned, which the kernel checks (an error, never a
  // misaligned swizzle atom).
  static constexpr int kSlack = kCtasPerSm == 2 ? 0 : 1024;
  static constexpr int kBytes = kBarOff + kBars * 8 + 16 + kSlack;
  static constexpr uint32_t kTmemCols = BN_ == 128 ? 512 : 256;
  static constexpr uint32_t kOCol = 2 * BN;  // S double buffer in columns [0, 2 BN), then O
  static_assert(BN_ == 64 || BN_ == 128, "key block of 64 or 128");
  static_assert(kBytes <= (kCtasPerSm == 2 ? 115712 : 232448), "shared memory per CTA");
  static_assert(2 * BN + D <= static_cast<int>(kTmemCols), "TMEM columns");
};

struct FmhaParams {
  void* out;
  int64_t o_sb, o_sh, o_ss;
  int seq_q, kv_rows, dense_kv, group, causal, q_s_inner, o_s_inner;
  const int64_t* positions;
  float scale_log2;
  unsigned* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Every lane waits (so each observes the completed phase), then the warp agrees.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const bool done = mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, done && *abort_flag == 0);
}

template <typename T, int D, int BNK, bool PT>
__global__ void __launch_bounds__(kFmhaThreads, FmhaLayout<D, BNK, PT>::kCtasPerSm)
    fmha_prefill_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
                        const FmhaParams p) {
  using L = FmhaLayout<D, BNK, PT>;
  constexpr int BM = L::BM, BN = L::BN, KST = L::KST, VST = L::VST;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  if (L::kSlack == 0 && (smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) set_device_error(p.err, kDevErrAttentionTimeout);
    return;  // uniform for the whole CTA: nothing was started
  }
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + KST;
  uint64_t* v_full = k_empty + KST;
  uint64_t* v_empty = v_full + VST;
  uint64_t* s_full = v_empty + VST;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* mma_done = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mb = gridDim.x - 1 - blockIdx.x;  // the longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / p.group;
  const int m0 = mb * BM;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    tma_prefetch_desc(&to);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // q, the cache rows and the positions come from earlier kernels
  pdl_wait();
  pdl_trigger();

  int kv_len = p.positions ? static_cast<int>(p.positions[b]) + p.seq_q : p.dense_kv;
  if (kv_len > p.kv_rows) {
    if (threadIdx.x == 0) set_device_error(p.err, kDevErrKvCapacity);
    kv_len = p.kv_rows;
  }
  const int off = kv_len - p.seq_q;  // bottom-right causal offset
  const int n_end = max(p.causal ? min(kv_len, m0 + BM + off) : kv_len, 0);
  const int nblocks = (n_end + BN - 1) / BN;

  if (warp == 0) {
    if (lane == 0 && nblocks > 0) {
      bool ok = true;
      mbar_arrive_expect_tx(q_full, L::kQBytes);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        if (p.q_s_inner) tma_load_4d(smem + L::kQOff + c * L::kBox, &tq, c * 64, m0, h, b, q_full);
        else tma_load_4d(smem + L::kQOff + c * L::kBox, &tq, c * 64, h, m0, b, q_full);
      }
      int k_issued = 0, v_issued = 0;
      auto load_k = [&](int j) -> bool {
        const int s = j % KST;
        if (!mbar_wait(&k_empty[s], ((j / KST) & 1) ^ 1) || *abort_flag) return false;
        mbar_arrive_expect_tx(&k_full[s], L::kKVBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(smem + L::kKOff + s * L::kKVBytes + c * BN * 128, &tk, c * 64, j * BN, kvh, b, &k_full[s]);
        k_issued = j + 1;
        return true;
      };
      auto load_v = [&](int j) -> bool {
        const int s = j % VST;
        if (!mbar_wait(&v_empty[s], ((j / VST) & 1) ^ 1) || *abort_flag) return false;
        mbar_arrive_expect_tx(&v_full[s], L::kKVBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(smem + L::kVOff + s * L::kKVBytes + c * BN * 128, &tv, c * 64, j * BN, kvh, b, &v_full[s]);
        v_issued = j + 1;
        return true;
      };
      // consumption order: K0, K1, V0, K2, V1, ...
      ok = load_k(0);
      for (int j = 0; j < nblocks && ok; ++j) {
        if (j + 1 < nblocks) ok = load_k(j + 1);
        if (ok) ok = load_v(j);
      }
      if (!ok) {
        set_device_error(p.err, kDevErrAttentionTimeout);
        *abort_flag = 1;
      }
      // No bulk copy may still be writing shared memory when the CTA exits.
      mbar_wait(q_full, 0);
      for (int j = max(0, k_issued - KST); j < k_issued; ++j) mbar_wait(&k_full[j % KST], (j / KST) & 1);
      for (int j = max(0, v_issued - VST); j < v_issued; ++j) mbar_wait(&v_full[j % VST], (j / VST) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && nblocks > 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(kBf16, BM, BN);
      constexpr uint32_t idesc_o = umma_idesc_f16_bmn(kBf16, BM, D);
      const uint32_t q_addr = smem_u32(smem + L::kQOff);
      const uint32_t p_addr = smem_u32(smem + L::kPOff);
      auto qk = [&](int j) -> bool {
        const int s = j % KST, sb = j & 1;
        if (!mbar_wait(&k_full[s], (j / KST) & 1)) return false;
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1) || *abort_flag) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kKOff + s * L::kKVBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(q_addr + (kk / 4) * L::kBox) + 2 * (kk % 4);
          const uint64_t bd = umma_desc_sw128(k_addr + (kk / 4) * (BN * 128)) + 2 * (kk % 4);
          umma_f16(tmem + static_cast<uint32_t>(sb * BN), ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[s]);
        umma_commit(&s_full[sb]);
        return true;
      };
      auto pv = [&](int j) -> bool {
        const int s = j % VST;
        if (!mbar_wait(p_full, j & 1)) return false;
        if (!mbar_wait(&v_full[s], (j / VST) & 1) || *abort_flag) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + L::kVOff + s * L::kKVBytes);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = umma_desc_mn_sw128(v_addr + kk * 16 * 128, BN * 128, 1024);
          if constexpr (PT) {
            // P_j over S_j's columns; the MMAs run in issue order, so S_{j+2}
            // (issued after this) cannot overwrite it before it is read
            umma_f16_ts(tmem + L::kOCol, tmem + static_cast<uint32_t>((j & 1) * BN + kk * 8), bd, idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
          } else {
            const uint64_t ad = umma_desc_sw128(p_addr + (kk / 4) * L::kBox) + 2 * (kk % 4);
            umma_f16(tmem + L::kOCol, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&v_empty[s]);
        umma_commit(o_done);
        return true;
      };
      bool ok = mbar_wait(q_full, 0);
      if (ok) ok = qk(0);
      for (int j = 0; j < nblocks && ok; ++j) {
        if (j + 1 < nblocks) ok = qk(j + 1);
        if (ok) ok = pv(j);
      }
      if (!ok) {
        set_device_error(p.err, kDevErrAttentionTimeout);
        *abort_flag = 1;
      }
      // every issued MMA has finished before the CTA releases tensor memory
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane = query row of the tile
    const int qrow = m0 + row;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    uint8_t* p_tile = smem + L::kPOff;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblocks; ++j) {
      const int sb = j & 1;
      if (!warp_wait(&s_full[sb], (j >> 1) & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tmem_ld_32x32b_x32(lane_base + static_cast<uint32_t>(sb * BN + c * 32),
                           *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);

      // mask: keys < lim are visible to this row
      const int key0 = j * BN;
      const bool full_block = key0 + BN <= kv_len && (!p.causal || key0 + BN - 1 <= m0 + off);
      if (!full_block) {
        const int lim = p.causal ? min(kv_len, qrow + off + 1) : kv_len;
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (key0 + i >= lim) sr[i] = __float_as_uint(-INFINITY);
      }
      // row maximum over 8 independent chains (short dependency chains: one
      // warp per scheduler, so latency is not hidden by other warps)
      float mc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mc[k] = max3(__uint_as_float(sr[2 * k]), __uint_as_float(sr[2 * k + 1]), -INFINITY);
#pragma unroll
      for (int i = 16; i < BN; i += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mc[k] = max3(mc[k], __uint_as_float(sr[i + 2 * k]), __uint_as_float(sr[i + 2 * k + 1]));
      const float mx = max3(max3(mc[0], mc[1], mc[2]), max3(mc[3], mc[4], mc[5]), fmaxf(mc[6], mc[7]));
      const float m_blk = mx * p.scale_log2;
      float alpha = 1.f;
      bool rescale_row = false;
      if (m_blk > m_used + kRescaleThreshold) {
        if (m_used != -INFINITY) {
          alpha = ex2(m_used - m_blk);
          rescale_row = true;
        }
        l *= alpha;
        m_used = m_blk;
      }
      bool waited = false;
      if (__any_sync(0xffffffffu, rescale_row)) {
        // O holds P_0 V_0 + ... + P_{j-1} V_{j-1}: wait for the last of them
        if (!warp_wait(o_done, (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        waited = true;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(lane_base + L::kOCol + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32x32b_x32(lane_base + L::kOCol + c, r);
        }
        tmem_st_wait();
      }
      // P = exp2(S * scale - m) (masked keys: exp2(-inf) = 0)
      const float neg = m_used == -INFINITY ? 0.f : -m_used;
      uint32_t pk[BN / 2];
      float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < BN; i += 2) {
        const float p0 = ex2(fmaf(__uint_as_float(sr[i]), p.scale_log2, neg));
        const float p1 = ex2(fmaf(__uint_as_float(sr[i + 1]), p.scale_log2, neg));
        rs[(i / 2) & 7] += p0 + p1;
        pk[i / 2] = pack_pair<T>(p0, p1);
      }
      l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      // P V_{j-1} must have consumed the shared P tile before it is rewritten
      // (a TMEM P goes over S_j, which no MMA reads)
      if (!PT && j > 0 && !waited) {
        if (!warp_wait(o_done, (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
      }
      // last block: zero V rows past the sequence that exist in memory
      if (j == nblocks - 1) {
        const int z0 = max(kv_len - key0, 0), z1 = min(BN, p.kv_rows - key0);
        if (z1 > z0) {
          if (!warp_wait(&v_full[j % VST], (j / VST) & 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* vt = smem + L::kVOff + (j % VST) * L::kKVBytes;
          const int per_box = (z1 - z0) * 8;  // 16-byte chunks per 64-column box
          for (int c = row; c < per_box * (D / 64); c += 128) {
            const int box = c / per_box, rem = c - box * per_box;
            *reinterpret_cast<uint4*>(vt + box * BN * 128 + (z0 + rem / 8) * 128 + (rem % 8) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
        }
      }
      if constexpr (PT) {
        // P row into this lane's S_j columns: BN 16-bit values in BN / 2 columns
#pragma unroll
        for (int c = 0; c < BN / 64; ++c)
          tmem_st_32x32b_x32(lane_base + static_cast<uint32_t>(sb * BN + c * 32),
                             *reinterpret_cast<const uint32_t(*)[32]>(&pk[c * 32]));
        tmem_st_wait();
        if (j == nblocks - 1) fence_proxy_async_smem();  // the zeroed V rows
      } else {
        // P row into the 128-byte-swizzled K-major tile (two 64-key boxes)
        uint8_t* prow = p_tile + row * 128;
        const int r7 = row & 7;
#pragma unroll
        for (int c = 0; c < BN / 8; ++c) {
          const int box = c >> 3, cc = c & 7;
          *reinterpret_cast<uint4*>(prow + box * L::kBox + ((cc ^ r7) << 4)) =
              make_uint4(pk[c * 4], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (!ok && lane == 0) {
      set_device_error(p.err, kDevErrAttentionTimeout);
      *abort_flag = 1;
    }
    // O / l as T into the Q tile's shared memory (the last Q K^T has completed),
    // in the same 128-byte-swizzled boxes, then one thread stores the tile by
    // TMA (rows past the sequence are outside the map and are not written).
    // Every softmax warp takes this path, abort or not, so the named barrier
    // below always completes.
    // Every MMA must have finished before O is read. The wait is on mma_done (one
    // phase, committed by the MMA thread after its last issue, abort included),
    // not on o_done: with P in tensor memory nothing here has waited for P V of
    // block nblocks-2, so o_done may still be two phases behind, and a parity
    // wait for phase nblocks-1 would then pass at once.
    bool have_o = ok && nblocks > 0;
    if (have_o && !warp_wait(mma_done, 0, abort_flag)) {
      if (lane == 0) set_device_error(p.err, kDevErrAttentionTimeout);
      have_o = false;
    }
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint8_t* orow = smem + L::kQOff + row * 128;
    const int r7 = row & 7;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t r[32];
      if (have_o) {
        tmem_ld_32x32b_x32(lane_base + L::kOCol + c, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 v;
        v.x = pack_pair<T>(__uint_as_float(r[q4 * 8 + 0]) * inv, __uint_as_float(r[q4 * 8 + 1]) * inv);
        v.y = pack_pair<T>(__uint_as_float(r[q4 * 8 + 2]) * inv, __uint_as_float(r[q4 * 8 + 3]) * inv);
        v.z = pack_pair<T>(__uint_as_float(r[q4 * 8 + 4]) * inv, __uint_as_float(r[q4 * 8 + 5]) * inv);
        v.w = pack_pair<T>(__uint_as_float(r[q4 * 8 + 6]) * inv, __uint_as_float(r[q4 * 8 + 7]) * inv);
        const int ch = ((c & 63) >> 3) + q4;  // 16-byte chunk of the 128-byte box row
        *reinterpret_cast<uint4*>(orow + (c >> 6) * L::kBox + ((ch ^ r7) << 4)) = v;
      }
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four softmax warps
    if (warp == 2 && lane == 0) {
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        if (p.o_s_inner) tma_store_4d(&to, smem + L::kQOff + c * L::kBox, c * 64, m0, h, b);
        else tma_store_4d(&to, smem + L::kQOff + c * L::kBox, c * 64, h, m0, b);
      }
      bulk_commit();
      bulk_wait_read();  // the tile stays in shared memory until the copy has read it
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

// ---- host ----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

}  // namespace

// 4-D map, dims[0] innermost (contiguous), strides in bytes for dims 1..3,
// 128-byte swizzle, out-of-range elements read as zero.
dli_status make_map_4d(CUtensorMap* map, const void* base, bool bf16, const uint64_t (&dims)[4],
                       const uint64_t (&strides)[3], const uint32_t (&box)[4]) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return fail(DLI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t s[3] = {strides[0], strides[1], strides[2]};
  const cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(base), d, s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  // A layout the tensor-map encoder rejects is served by the mma.sync kernel.
  if (r != CUDA_SUCCESS)
    return fail(DLI_ERR_UNSUPPORTED, "attention: cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
  return DLI_OK;
}

namespace {

template <typename T, int D, int BNK, bool PT>
dli_status launch_fmha(const FmhaArgs& a, cudaStream_t stream) {
  using L = FmhaLayout<D, BNK, PT>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap tq, tk, tv, to;
  const bool s_inner = a.q_ss <= a.q_sh;
  const uint64_t qd[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(s_inner ? a.seq_q : a.hq),
                          static_cast<uint64_t>(s_inner ? a.hq : a.seq_q), static_cast<uint64_t>(a.batch)};
  const uint64_t qs[3] = {static_cast<uint64_t>((s_inner ? a.q_ss : a.q_sh) * 2),
                          static_cast<uint64_t>((s_inner ? a.q_sh : a.q_ss) * 2), static_cast<uint64_t>(a.q_sb * 2)};
  const uint32_t qb[4] = {64u, s_inner ? 128u : 1u, s_inner ? 1u : 128u, 1u};
  dli_status st = make_map_4d(&tq, a.q, kBf16, qd, qs, qb);
  if (st != DLI_OK) return st;
  const int64_t rows = a.k_sh / D;
  const uint64_t kd[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(rows), static_cast<uint64_t>(a.hkv),
                          static_cast<uint64_t>(a.batch)};
  const uint64_t ks[3] = {static_cast<uint64_t>(D * 2), static_cast<uint64_t>(a.k_sh * 2),
                          static_cast<uint64_t>(a.k_sb * 2)};
  const uint32_t kb[4] = {64u, static_cast<uint32_t>(L::BN), 1u, 1u};
  st = make_map_4d(&tk, a.k, kBf16, kd, ks, kb);
  if (st != DLI_OK) return st;
  st = make_map_4d(&tv, a.v, kBf16, kd, ks, kb);
  if (st != DLI_OK) return st;
  FmhaParams p{};
  p.out = a.out;
  p.o_sb = a.o_sb;
  p.o_sh = a.o_sh;
  p.o_ss = a.o_ss;
  p.seq_q = a.seq_q;
  p.kv_rows = static_cast<int>(rows);
  p.dense_kv = a.dense_kv;
  p.group = a.hq / a.hkv;
  p.causal = a.causal;
  p.q_s_inner = s_inner ? 1 : 0;
  // the output tile goes out through its own map (the output may be laid out
  // differently from q)
  const bool o_inner = a.o_ss <= a.o_sh;
  const uint64_t od[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(o_inner ? a.seq_q : a.hq),
                          static_cast<uint64_t>(o_inner ? a.hq : a.seq_q), static_cast<uint64_t>(a.batch)};
  const uint64_t os[3] = {static_cast<uint64_t>((o_inner ? a.o_ss : a.o_sh) * 2),
                          static_cast<uint64_t>((o_inner ? a.o_sh : a.o_ss) * 2), static_cast<uint64_t>(a.o_sb * 2)};
  const uint32_t ob[4] = {64u, o_inner ? 128u : 1u, o_inner ? 1u : 128u, 1u};
  st = make_map_4d(&to, a.out, kBf16, od, os, ob);
  if (st != DLI_OK) return st;
  p.o_s_inner = o_inner ? 1 : 0;
  p.positions = a.positions;
  p.scale_log2 = a.scale_log2;
  p.err = device_error_word();
  auto kern = fmha_prefill_kernel<T, D, BNK, PT>;
  st = ensure_smem(reinterpret_cast<const void*>(kern), L::kBytes, "attention prefill (tcgen05)");
  if (st != DLI_OK) return st;
  dim3 grid(static_cast<unsigned>(ceil_div(a.seq_q, L::BM)), static_cast<unsigned>(a.hq),
            static_cast<unsigned>(a.batch));
  launch_pdl(kern, grid, dim3(kFmhaThreads), L::kBytes, stream, tq, tk, tv, to, p);
  return check_launch("attention prefill (tcgen05)");
}

}  // namespace

// DLI_SM100_ATTN_FMHA: 0 = prefill on the mma.sync kernel, 1 (default) = this
// kernel where the layout allows, 2 = this kernel or an error (tests use it to
// prove which kernel ran).
static int fmha_mode() {
  static const int mode = tuning_knob("ATTN_FMHA", 1);
  return mode;
}

bool fmha_required() { return fmha_mode() == 2; }

bool fmha_supported(const FmhaArgs& a, dli_dtype dtype) {
  if (fmha_mode() == 0) return false;
  if (dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16) return false;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  if (a.batch <= 0 || a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv != 0 || a.seq_q <= 0) return false;
  if (a.batch > 65535 || a.hq > 65535) return false;
  for (const void* ptr : {a.q, a.k, a.v, static_cast<const void*>(a.out)})
    if (!aligned(ptr, 16)) return false;
  // TMA strides and 16-byte output vectors: every stride a multiple of 8 elements
  for (int64_t s : {a.q_sb, a.q_sh, a.q_ss, a.o_sb, a.o_sh, a.o_ss, a.k_sb, a.k_sh})
    if (s <= 0 || s % 8 != 0) return false;
  if (a.k_sh % a.head_dim != 0) return false;
  // the batch stride is the outermost (4-D maps list dims by increasing stride)
  if (a.q_sb < std::max(a.q_sh, a.q_ss) || a.o_sb < std::max(a.o_sh, a.o_ss) || a.k_sb < a.k_sh) return false;
  if (std::min(a.q_sh, a.q_ss) < a.head_dim || std::min(a.o_sh, a.o_ss) < a.head_dim || a.k_sh / a.head_dim < 1)
    return false;
  if (a.k_sh / a.head_dim > (1ll << 30)) return false;
  return true;
}

// DLI_SM100_ATTN_FMHA_BN: keys per block, 64 (default: two CTAs per SM) or 128
// (one). Measured at the Qwen2-7B prefill launch (32 x 2048, 28/4 heads): 1.39
// against 1.70 ms.
static int fmha_block_keys() {
  static const int bn = tuning_knob("ATTN_FMHA_BN", 64) == 128 ? 128 : 64;
  return bn;
}

// DLI_SM100_ATTN_FMHA_P: where P = exp2(S * scale - m) is staged for O += P V:
// 1 (default) tensor memory, over the S buffer; 0 a swizzled shared-memory tile.
static bool fmha_p_in_tmem() {
  static const bool tm = tuning_knob("ATTN_FMHA_P", 1) != 0;
  return tm;
}

template <int BNK, bool PT>
dli_status run_fmha_bn(const FmhaArgs& a, dli_dtype dtype, cudaStream_t stream) {
  if (dtype == DLI_DTYPE_BF16)
    return a.head_dim == 64 ? launch_fmha<__nv_bfloat16, 64, BNK, PT>(a, stream)
                            : launch_fmha<__nv_bfloat16, 128, BNK, PT>(a, stream);
  return a.head_dim == 64 ? launch_fmha<__half, 64, BNK, PT>(a, stream)
                          : launch_fmha<__half, 128, BNK, PT>(a, stream);
}

dli_status run_fmha_prefill(const FmhaArgs& a, dli_dtype dtype, cudaStream_t stream) {
  if (fmha_p_in_tmem())
    return fmha_block_keys() == 64 ? run_fmha_bn<64, true>(a, dtype, stream) : run_fmha_bn<128, true>(a, dtype, stream);
  return fmha_block_keys() == 64 ? run_fmha_bn<64, false>(a, dtype, stream) : run_fmha_bn<128, false>(a, dtype, stream);
}

}  // namespace dli_sm100
