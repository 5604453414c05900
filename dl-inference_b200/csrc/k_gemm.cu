// GEMM kernels behind linear, matmul and conv2d.
//
// tcgen05 path (bf16/f16 operands, fp32 accumulation) — a warp-specialised TN
// GEMM  D[i, j] = sum_k A[i, k] * B[j, k]  with both operands K-major (the
// nn.Linear layout x[M,K], w[N,K]):
//   warp 0     TMA producer: 128x64 A box + BNx64 B box per stage, 128-byte
//              swizzle, STAGES-deep mbarrier ring (full/empty);
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN,
//              K=16 per instruction, 4 per stage), tcgen05.commit frees a stage;
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time from the warp's TMEM
//              lane quarter, bias add, convert, store.
// Decode-sized problems (few activation rows) run swap-AB: A = weights (rows N
// fill the 128-row MMA), B = activations (BN = rows rounded up to 16), so the
// weight matrix streams through HBM exactly once; when the tiles cannot fill the
// GPU, K is split over a thread-block cluster of S CTAs per tile, whose fp32
// partial tiles are reduced through distributed shared memory in rank order.
// Prefill-sized problems run A = activations, B = weights with BN = 128/256 and
// grouped tile rasterisation for L2 reuse.
//
// SIMT path: exact-fp32 FFMA tiles for fp32 tensors (the reference kernel,
// python/dli_ops/aot/linear/kernel.py:24-38, runs fp32 tl.dot as TF32; the
// accuracy target here is fp32), and for shapes TMA cannot address.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "gemm.cuh"
#include "exchange.cuh"
#include "tcgen05.cuh"

namespace dli_sm100 {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kGroupI = 8;

// kPush (tile widths <= 64, the decode tiles): split-K partials are pushed into a
// dedicated receive buffer of the owning cluster rank (kRecvRows rows of BN + 4
// floats: S ranks x R rows never exceed 128 + 2 * 7); wider tiles stage their
// partial in the idle operand ring and pull.
template <int BN, int STAGES>
struct TcLayout {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr bool kPush = BN <= 64;
  static constexpr int kRecvRows = kBM + 16;
  static constexpr int kRecvOff = STAGES * kStageBytes;
  static constexpr int kRecvBytes = kPush ? kRecvRows * (BN + 4) * 4 : 0;
  static constexpr int kBarOffset = kRecvOff + kRecvBytes;
  // full[STAGES], empty[STAGES], acc_full, red_full
  static constexpr int kBytes = kBarOffset + (2 * STAGES + 2) * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzle atoms need 1 KiB alignment");
  // the pull reduction stages the partial tile [128][BN + 4] fp32 in the idle operand ring
  static_assert(kBM * (BN + 4) * 4 <= STAGES * kStageBytes, "split-K staging must fit the operand ring");
};

// Owner of accumulator row `row` under a push reduction over S cluster ranks, and
// its row index in the owner's receive slot. Row-per-rank layouts: rank r owns
// rows [r*R, (r+1)*R), R = ceil(128/S). kEpiGluT: rank r owns gate rows
// [r*Rg, (r+1)*Rg) of 0..63, Rg = ceil(64/S), and the matching up rows (+64),
// stored after its Rg gate rows.
// kEpiExchange, kEpiQkvRotary: R = 2*ceil(64/S), even, so each rank owns whole
// feature pairs.
__device__ __host__ __forceinline__ int push_rows_per_rank(int epilogue, int S) {
  return (epilogue == kEpiExchange || epilogue == kEpiQkvRotary) ? 2 * ((64 + S - 1) / S) : (kBM + S - 1) / S;
}
__device__ __forceinline__ void push_owner(int epilogue, int S, int row, int& owner, int& lidx) {
  if (epilogue == kEpiGluT) {
    const int rg = (64 + S - 1) / S, g = row & 63;
    owner = g / rg;
    lidx = (g - owner * rg) + (row >> 6) * rg;
  } else {
    const int r = push_rows_per_rank(epilogue, S);
    owner = row / r;
    lidx = row - owner * r;
  }
}
// Receive-slot height (rows per sender) and the rows this rank owns.
__device__ __host__ __forceinline__ int push_slot_rows(int epilogue, int S) {
  return epilogue == kEpiGluT ? 2 * ((64 + S - 1) / S) : push_rows_per_rank(epilogue, S);
}
__device__ __host__ __forceinline__ int push_my_rows(int epilogue, int S, int rank) {
  if (epilogue == kEpiGluT) {
    const int rg = (64 + S - 1) / S;
    return 2 * max(0, min(rg, 64 - rank * rg));
  }
  const int r = push_rows_per_rank(epilogue, S);
  return max(0, min(r, kBM - rank * r));
}

struct TcParams {
  int rows_a, rows_b;
  int tiles_i, tiles_j;
  int kblocks, splits;  // splits > 1: the grid's y CTAs of a tile form one cluster
  int epilogue;
  int64_t ldo, ohw;
  int out_vec;  // output base is 16-byte aligned
  int const_a;  // operand A is read-only weights: its first tiles load before pdl_wait
  int const_b;  // same for operand B
  int glu_cols; // SwiGLU epilogues: valid output columns (the intermediate size)
  int out_f32;  // RowMajor / Transposed: the output is float32 (operands stay T)
  int b_mn;     // operand B is MN-major: [K, rows_b] with rows_b contiguous (matmul)
  int bias_f32; // out_f32 epilogues: the bias is float32 (fp32 GEMM), else T
  // kEpiExchange: the group's exchange buffers as mapped here, this rank, and their geometry
  char* xbuf[kExchangeMaxRanks];
  int xtp, xrank;
  int64_t xmax_rows, xrow_words;
  // kEpiQkvRotary: tables [table_rows, pairs], positions [B], outputs, geometry
  const float* rot_cos;
  const float* rot_sin;
  const int64_t* rot_pos;
  void* rot_q;
  void* rot_k;
  void* rot_v;
  int rot_hq, rot_hkv, rot_d, rot_seq;
  int64_t rot_pairs, rot_rows, rot_cap;
  // stream-K (tcgen05_gemm_streamk_kernel): partial tiles [ctas][2][128][BN] fp32
  // and one arrival counter per tile, zero between calls
  float* sk_part;
  int* sk_count;
  const void* bias;
  void* out;
  unsigned* err;
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_i, int tiles_j, int& ti, int& tj) {
  const int per_group = kGroupI * tiles_j;
  const int g = tile / per_group;
  const int first = g * kGroupI;
  const int gsize = min(tiles_i - first, kGroupI);
  const int r = tile - g * per_group;
  ti = first + r % gsize;
  tj = r / gsize;
}

// Operand B of one K block (BN rows x kBK). K-major B ([rows_b, K]) is one box;
// MN-major B ([K, rows_b]) is BN/64 boxes, each a 128B-swizzled panel of kBK K
// rows x 64 consecutive j (the host never pairs MN-major B with BN < 64).
template <int BN>
__device__ __forceinline__ void load_b_block(uint8_t* dst, const CUtensorMap* map, int kb, int tj, int b_mn,
                                             uint64_t* bar) {
  if (b_mn) {
#pragma unroll
    for (int c = 0; c < BN / 64; ++c) tma_load_2d(dst + c * 64 * kBK * 2, map, tj * BN + c * 64, kb * kBK, bar);
  } else {
    tma_load_2d(dst, map, kb * kBK, tj * BN, bar);
  }
}

// Shared-memory descriptor of operand B at K step kk (16 elements) of a block:
// K-major advances 32 bytes inside the swizzle atom; MN-major advances 16 K rows
// (2 KiB), with the 64-column panels kBK * 128 bytes apart (leading offset) and
// 8-row groups 1 KiB apart (stride offset).
__device__ __forceinline__ uint64_t b_block_desc(uint32_t b_addr, int kk, int b_mn) {
  return b_mn ? umma_desc_mn_sw128(b_addr + kk * 16 * 128, 64 * kBK * 2, 1024) : umma_desc_sw128(b_addr) + 2 * kk;
}

// Writes n (<= 32) accumulator values of D row `gi`, columns jc.. through the
// epilogue mapping, adding the bias.
template <typename T>
__device__ __forceinline__ void store_vals(const TcParams& p, int64_t gi, int jc, const float* v,
                                           int n) {
  const T* bias = static_cast<const T*>(p.bias);
  T* out = static_cast<T*>(p.out);
  if (gi >= p.rows_a) return;
  if (p.out_f32) {  // fp32 output (logits): the accumulator is stored unrounded
    float* outf = static_cast<float*>(p.out);
    const float* biasf = static_cast<const float*>(p.bias);
    const bool tr = p.epilogue == kEpiTransposed;
    auto bias_at = [&](int64_t i) { return !bias ? 0.f : p.bias_f32 ? biasf[i] : to_f32(bias[i]); };
    const float bt = tr ? bias_at(gi) : 0.f;
    for (int k = 0; k < n && jc + k < p.rows_b; ++k) {
      const float bv = tr ? bt : bias_at(jc + k);
      outf[tr ? static_cast<int64_t>(jc + k) * p.ldo + gi : gi * p.ldo + jc + k] = v[k] + bv;
    }
    return;
  }
  if (p.epilogue == kEpiRowMajor) {
    T* dst = out + gi * p.ldo + jc;
    if (n == 32 && p.out_vec && jc + 32 <= p.rows_b && (p.ldo % 8) == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        Vec16<T> pack;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int k = q * 8 + e;
          const float bv = bias ? to_f32(bias[jc + k]) : 0.f;
          pack.e[e] = from_f32<T>(v[k] + bv);
        }
        store16(dst + q * 8, pack);
      }
    } else {
      for (int k = 0; k < n && jc + k < p.rows_b; ++k) {
        const float bv = bias ? to_f32(bias[jc + k]) : 0.f;
        dst[k] = from_f32<T>(v[k] + bv);
      }
    }
  } else if (p.epilogue == kEpiTransposed) {
    const float bv = bias ? to_f32(bias[gi]) : 0.f;
    for (int k = 0; k < n && jc + k < p.rows_b; ++k)
      out[static_cast<int64_t>(jc + k) * p.ldo + gi] = from_f32<T>(v[k] + bv);
  } else {  // kEpiNchw
    const int64_t img = gi / p.ohw, pix = gi - img * p.ohw;
    for (int k = 0; k < n && jc + k < p.rows_b; ++k) {
      const float bv = bias ? to_f32(bias[jc + k]) : 0.f;
      out[(img * p.rows_b + jc + k) * p.ohw + pix] = from_f32<T>(v[k] + bv);
    }
  }
}

// SwiGLU of one gate/up accumulator pair: silu(g) * u from the fp32
// accumulators, rounded to T once (the unfused graph rounds the gate and up
// outputs, the silu and the product: four bf16 roundings instead of one).
template <typename T>
__device__ __forceinline__ T glu_val(float g, float u) {
  return from_f32<T>(g / (1.0f + expf(-g)) * u);
}

// kEpiGluT: n (<= 32) consecutive tokens j0.. of gate row `grow` (0..63) of tile ti.
template <typename T>
__device__ __forceinline__ void store_glu_t(const TcParams& p, int ti, int grow, int j0, const float* g,
                                            const float* u, int n) {
  const int64_t col = static_cast<int64_t>(ti) * 64 + grow;
  if (col >= p.glu_cols) return;
  T* out = static_cast<T*>(p.out);
  for (int k = 0; k < n && j0 + k < p.rows_b; ++k) out[static_cast<int64_t>(j0 + k) * p.ldo + col] = glu_val<T>(g[k], u[k]);
}

__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Epilogue of one finished (un-split) accumulator tile for the layouts whose D
// row lives in one thread: this thread's row `gi`, TMEM columns from `tbase`
// (its lane quarter), tile column origin j0. RowMajor / Transposed / Nchw go
// through store_vals; kEpiGlu pairs gate columns c..c+63 with up columns
// c+64..c+127 of every 128-column block.
template <typename T, int BN>
__device__ __forceinline__ void epilogue_tile(const TcParams& p, uint32_t tbase, int64_t gi, int j0) {
  if (p.epilogue == kEpiGlu) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 128) {
#pragma unroll 1
      for (int h = 0; h < 64; h += 32) {
        uint32_t rg[32], ru[32];
        tmem_ld_32x32b_x32(tbase + c + h, rg);
        tmem_ld_32x32b_x32(tbase + c + 64 + h, ru);
        tmem_ld_wait();
        const int64_t oc = (static_cast<int64_t>(j0) + c) / 2 + h;
        if (gi < p.rows_a && oc < p.glu_cols) {
          T* dst = static_cast<T*>(p.out) + gi * p.ldo + oc;
          if (p.out_vec && (p.ldo % 8) == 0 && oc + 32 <= p.glu_cols) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              Vec16<T> pack;
#pragma unroll
              for (int e = 0; e < 8; ++e)
                pack.e[e] = glu_val<T>(__uint_as_float(rg[q * 8 + e]), __uint_as_float(ru[q * 8 + e]));
              store16(dst + q * 8, pack);
            }
          } else {
            for (int k = 0; k < 32 && oc + k < p.glu_cols; ++k)
              dst[k] = glu_val<T>(__uint_as_float(rg[k]), __uint_as_float(ru[k]));
          }
        }
      }
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tbase + c, r);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(r[k]);
    if (j0 + c < p.rows_b) store_vals<T>(p, gi, j0 + c, v, 32);
  }
}

// Epilogue warps (2-5) of a one-tile CTA: wait for the accumulator, then store
// the tile (un-split) or stage its fp32 partial in shared memory for the cluster
// reduction (split-K). `smem` is the CTA's idle operand ring.
template <typename T, int BN>
__device__ __forceinline__ void tile_epilogue_warps(const TcParams& p, uint8_t* smem, uint32_t tmem_base,
                                                    uint64_t* acc_full, volatile int* flags, int ti, int tj,
                                                    int warp, int lane) {
  // Epilogue: warp w may only touch TMEM lanes 32*(w%4) .. 32*(w%4)+31.
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int64_t gi = static_cast<int64_t>(ti) * kBM + row;
  const int j0 = tj * BN;
  const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  if (!mbar_wait(acc_full, 0)) {
    set_device_error(p.err, kDevErrGemmTimeout);
    flags[0] = 1;
  }
  tc_fence_after();
  epilogue_bar();  // every epilogue warp sees the same abort flag
  const bool aborted = flags[0] != 0;
  if (!aborted && p.splits == 1 && p.epilogue == kEpiGluT) {
    // gate rows live in TMEM lanes 0-63 (quarters 0, 1), up rows in lanes 64-127:
    // the up quarters pass their values through shared memory (the idle ring)
    float* xch = reinterpret_cast<float*>(smem);  // [64][33]
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + c, r);
      tmem_ld_wait();
      if (quarter >= 2) {
#pragma unroll
        for (int k = 0; k < 32; ++k) xch[(row - 64) * 33 + k] = __uint_as_float(r[k]);
      }
      epilogue_bar();
      const int64_t col = static_cast<int64_t>(ti) * 64 + row;
      if (quarter < 2 && col < p.glu_cols) {
        T* out = static_cast<T*>(p.out) + col;
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (j0 + c + k < p.rows_b)
            out[static_cast<int64_t>(j0 + c + k) * p.ldo] = glu_val<T>(__uint_as_float(r[k]), xch[row * 33 + k]);
      }
      epilogue_bar();
    }
  } else if (!aborted && p.splits == 1) {
    epilogue_tile<T, BN>(p, tbase, gi, j0);
  } else if (p.splits > 1) {
    // Split-K: stage this CTA's fp32 partial tile in its own shared memory
    // (the operand ring is idle: every load was consumed before acc_full).
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int k = 0; k < 32; k += 4)
        *reinterpret_cast<float4*>(red + row * (BN + 4) + c + k) =
            make_float4(aborted ? 0.f : __uint_as_float(r[k]), aborted ? 0.f : __uint_as_float(r[k + 1]),
                        aborted ? 0.f : __uint_as_float(r[k + 2]), aborted ? 0.f : __uint_as_float(r[k + 3]));
    }
  }
}

// Split-K tail, run by every thread of every CTA of the tile's cluster after
// the partials were staged (tile_epilogue_warps) and the CTA synchronised.
template <typename T, int BN, int kThreads = kGemmThreads>
__device__ __forceinline__ void tile_cluster_reduce(const TcParams& p, uint8_t* smem, int ti, int tj, int split) {
  // The K-splits of this tile form one thread-block cluster (ranks 0..S-1 along
  // y). After the cluster barrier every partial is visible through distributed
  // shared memory; CTA `split` sums rows [split*R, (split+1)*R) of all S
  // partials in rank order (deterministic) and writes them. The second barrier
  // keeps every CTA's shared memory alive until all ranks finished reading.
  cluster_sync();
  const int S = p.splits;
  const uint32_t red_local = smem_u32(smem);
  if (p.epilogue == kEpiGluT) {
    // each rank reduces gate rows [split*R, ...) of 0..63 and their up rows (+64)
    const int R = (64 + S - 1) / S;
    const int quads = R * (BN / 4);
    for (int q = threadIdx.x; q < quads; q += kThreads) {
      const int rr = split * R + q % R;
      const int cq = (q / R) * 4;
      if (rr >= 64) continue;
      const uint32_t og = static_cast<uint32_t>((rr * (BN + 4) + cq) * 4);
      const uint32_t ou = static_cast<uint32_t>(((rr + 64) * (BN + 4) + cq) * 4);
      float4 pg[8], pu[8];
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        if (s2 < S) {
          pg[s2] = ld_dsmem_f4(mapa_shared(red_local + og, s2));
          pu[s2] = ld_dsmem_f4(mapa_shared(red_local + ou, s2));
        }
      }
      float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        if (s2 < S) {
          g[0] += pg[s2].x; g[1] += pg[s2].y; g[2] += pg[s2].z; g[3] += pg[s2].w;
          u[0] += pu[s2].x; u[1] += pu[s2].y; u[2] += pu[s2].z; u[3] += pu[s2].w;
        }
      }
      if (tj * BN + cq < p.rows_b) store_glu_t<T>(p, ti, rr, tj * BN + cq, g, u, 4);
    }
  }
  const int R = (kBM + S - 1) / S;  // rows reduced by each rank (the last may get fewer)
  const int quads = p.epilogue == kEpiGluT ? 0 : R * (BN / 4);
  for (int q = threadIdx.x; q < quads; q += kThreads) {
    const int rr = split * R + q % R;  // consecutive threads: consecutive rows
    const int cq = (q / R) * 4;
    if (rr >= kBM) continue;
    const uint32_t off = static_cast<uint32_t>((rr * (BN + 4) + cq) * 4);
    // issue every rank's load before the first add: one DSMEM round trip, not S
    float4 part[8];
#pragma unroll
    for (int s = 0; s < 8; ++s)
      if (s < S) part[s] = ld_dsmem_f4(mapa_shared(red_local + off, s));
    float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      if (s < S) {
        v[0] += part[s].x;
        v[1] += part[s].y;
        v[2] += part[s].z;
        v[3] += part[s].w;
      }
    }
    const int64_t gi = static_cast<int64_t>(ti) * kBM + rr;
    if (tj * BN + cq < p.rows_b) store_vals<T>(p, gi, tj * BN + cq, v, 4);
  }
  cluster_sync();
}

// Split-K by push (epilogue warps 2-5): wait for the accumulator, then send each
// accumulator row to the cluster rank that owns it, into slot `split` of that
// rank's receive buffer, with st.async completing bytes on the owner's
// red_full mbarrier (the own rank's rows are plain shared stores). Every rank
// sends all of its rows, zeros after an abort, so no receiver waits for bytes
// that never come. The owners' barriers were initialised before the
// cluster-barrier arrival at kernel start; cluster_wait() makes that visible.
template <typename T, int BN, int STAGES>
__device__ __forceinline__ void tile_push_partial(const TcParams& p, uint8_t* smem, uint32_t tmem_base,
                                                  uint64_t* acc_full, uint64_t* red_full, volatile int* flags,
                                                  int split, int warp, int lane) {
  using L = TcLayout<BN, STAGES>;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  if (!mbar_wait(acc_full, 0)) {
    set_device_error(p.err, kDevErrGemmTimeout);
    flags[0] = 1;
  }
  tc_fence_after();
  epilogue_bar();  // every epilogue warp sees the same abort flag
  const bool aborted = flags[0] != 0;
  int owner, lidx;
  push_owner(p.epilogue, p.splits, row, owner, lidx);
  const int slot_rows = push_slot_rows(p.epilogue, p.splits);
  const uint32_t dst_local = smem_u32(smem + L::kRecvOff) +
                             static_cast<uint32_t>(((split * slot_rows + lidx) * (BN + 4)) * 4);
  const uint32_t dst = mapa_shared(dst_local, static_cast<uint32_t>(owner));
  const uint32_t bar = mapa_shared(smem_u32(red_full), static_cast<uint32_t>(owner));
  cluster_wait();
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tbase + c, r);
    tmem_ld_wait();
#pragma unroll
    for (int k = 0; k < 32 && c + k < BN; k += 4) {
      const float4 v = aborted ? make_float4(0.f, 0.f, 0.f, 0.f)
                               : make_float4(__uint_as_float(r[k]), __uint_as_float(r[k + 1]),
                                             __uint_as_float(r[k + 2]), __uint_as_float(r[k + 3]));
      if (owner == split)
        *reinterpret_cast<float4*>(smem + L::kRecvOff + ((split * slot_rows + lidx) * (BN + 4) + c + k) * 4) = v;
      else
        st_async_f4(dst + static_cast<uint32_t>((c + k) * 4), v, bar);
    }
  }
}

// Split-K by push, all threads after a CTA barrier: wait until every peer's rows
// arrived (bounded; longer than any sender's own bounded waits), then sum this
// rank's rows over the S slots in rank order (deterministic) and store them.
template <typename T, int BN, int STAGES, int kThreads = kGemmThreads>
__device__ __forceinline__ void tile_push_reduce(const TcParams& p, uint8_t* smem, uint64_t* red_full, int ti, int tj,
                                                 int split) {
  using L = TcLayout<BN, STAGES>;
  const int S = p.splits;
  const int slot_rows = push_slot_rows(p.epilogue, S);
  const int mine = push_my_rows(p.epilogue, S, split);
  if (!mbar_wait(red_full, 0, 8000000000ull)) {
    if (threadIdx.x == 0) set_device_error(p.err, kDevErrGemmTimeout);
    return;
  }
  const float* recv = reinterpret_cast<const float*>(smem + L::kRecvOff);
  if (p.epilogue == kEpiGluT) {
    const int rg = mine / 2, rgs = slot_rows / 2;
    const int quads = rg * (BN / 4);
    for (int q = threadIdx.x; q < quads; q += kThreads) {
      const int lg = q % rg, cq = (q / rg) * 4;
      float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s2 = 0; s2 < S; ++s2) {
        const float4 a = *reinterpret_cast<const float4*>(recv + (s2 * slot_rows + lg) * (BN + 4) + cq);
        const float4 b = *reinterpret_cast<const float4*>(recv + (s2 * slot_rows + lg + rgs) * (BN + 4) + cq);
        g[0] += a.x; g[1] += a.y; g[2] += a.z; g[3] += a.w;
        u[0] += b.x; u[1] += b.y; u[2] += b.z; u[3] += b.w;
      }
      if (tj * BN + cq < p.rows_b) store_glu_t<T>(p, ti, split * rgs + lg, tj * BN + cq, g, u, 4);
    }
    return;
  }
  const int quads = mine * (BN / 4);
  if (p.epilogue == kEpiExchange) {
    // rows = output features, columns = tokens; a word holds features (f, f+1)
    // of one token: the even row's thread packs its value with its neighbour's
    // (mine and the rank's first row are even, so the pair is lanes q, q ^ 1)
    // and stores the word, at the token row's next epoch, into every rank's buffer
    const uint32_t* epochs = reinterpret_cast<const uint32_t*>(p.xbuf[p.xrank]);
    const T* bias = static_cast<const T*>(p.bias);
    for (int base = 0; base < quads; base += kThreads) {  // the same trip count in every lane
      const int q = base + static_cast<int>(threadIdx.x);
      const bool act = q < quads;
      const int lr = act ? q % mine : 0, cq = act ? (q / mine) * 4 : 0;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (act) {
        for (int s2 = 0; s2 < S; ++s2) {
          const float4 a = *reinterpret_cast<const float4*>(recv + (s2 * slot_rows + lr) * (BN + 4) + cq);
          v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
        }
      }
      const int64_t f = static_cast<int64_t>(ti) * kBM + split * slot_rows + lr;  // output feature
      const bool live = act && f < p.rows_a;
      const float bv = (live && bias) ? to_f32(bias[f]) : 0.f;
      uint32_t h[4], other[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const T x = from_f32<T>(v[k] + bv);
        h[k] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&x));
        other[k] = __shfl_xor_sync(0xffffffffu, h[k], 1);
      }
      if (live && (lr & 1) == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int t = tj * BN + cq + k;  // token = exchange row
          if (t >= p.rows_b) break;
          const uint32_t e = epochs[t] + 1u;
          for (int dst = 0; dst < p.xtp; ++dst)
            exchange_store_word(exchange_row_words(p.xbuf[dst], p.xmax_rows, p.xrow_words, p.xtp,
                                                   static_cast<int>(e & 1u), p.xrank, t) + f / 2,
                                h[k] | (other[k] << 16), e);
        }
      }
    }
    return;
  }
  if (p.epilogue == kEpiQkvRotary) {
    // rows = features of q|k|v, columns = tokens. Each value is rounded to T
    // first (the projection's output), then the even/odd features of a rotated
    // pair (lanes q, q ^ 1) combine with the table entry of the token's
    // position exactly as the separate rotary kernel computes them.
    const T* bias = static_cast<const T*>(p.bias);
    const int D = p.rot_d;
    for (int base = 0; base < quads; base += kThreads) {  // the same trip count in every lane
      const int q = base + static_cast<int>(threadIdx.x);
      const bool act = q < quads;
      const int lr = act ? q % mine : 0, cq = act ? (q / mine) * 4 : 0;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (act) {
        for (int s2 = 0; s2 < S; ++s2) {
          const float4 a = *reinterpret_cast<const float4*>(recv + (s2 * slot_rows + lr) * (BN + 4) + cq);
          v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
        }
      }
      const int f = ti * kBM + split * slot_rows + lr;  // feature of q|k|v
      const bool live = act && f < p.rows_a;
      const float bv = (live && bias) ? to_f32(bias[f]) : 0.f;
      float x[4], xo[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        x[k] = round_through<T>(v[k] + bv);
        xo[k] = __shfl_xor_sync(0xffffffffu, x[k], 1);
      }
      if (!live) continue;
      const int head = f / D, d = f - head * D, pair = d >> 1;
      const bool even = (d & 1) == 0;
      const bool rotated = head < p.rot_hq + p.rot_hkv && pair < p.rot_pairs;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int t = tj * BN + cq + k;  // token b * S + s
        if (t >= p.rows_b) break;
        const int b = t / p.rot_seq, sq = t - b * p.rot_seq;
        const int64_t pos = p.rot_pos[b] + sq;
        float y = x[k];
        if (rotated) {
          if (pos >= 0 && pos < p.rot_rows) {
            const float c = p.rot_cos[pos * p.rot_pairs + pair], sn = p.rot_sin[pos * p.rot_pairs + pair];
            const float a = even ? x[k] : xo[k], bb = even ? xo[k] : x[k];
            y = even ? a * c - bb * sn : a * sn + bb * c;
          } else {
            set_device_error(p.err, kDevErrRotaryPosition);
          }
        }
        const T o = from_f32<T>(y);
        if (head < p.rot_hq) {
          static_cast<T*>(p.rot_q)[(static_cast<int64_t>(t) * p.rot_hq + head) * D + d] = o;
        } else if (pos >= 0 && pos < p.rot_cap) {
          const bool is_k = head < p.rot_hq + p.rot_hkv;
          const int kvh = is_k ? head - p.rot_hq : head - p.rot_hq - p.rot_hkv;
          static_cast<T*>(is_k ? p.rot_k : p.rot_v)[((static_cast<int64_t>(b) * p.rot_hkv + kvh) * p.rot_cap + pos) * D +
                                                  d] = o;
        } else {
          set_device_error(p.err, kDevErrKvCapacity);
        }
      }
    }
    return;
  }
  for (int q = threadIdx.x; q < quads; q += kThreads) {
    const int lr = q % mine, cq = (q / mine) * 4;  // consecutive threads: consecutive rows
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s2 = 0; s2 < S; ++s2) {
      const float4 a = *reinterpret_cast<const float4*>(recv + (s2 * slot_rows + lr) * (BN + 4) + cq);
      v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
    }
    const int64_t gi = static_cast<int64_t>(ti) * kBM + split * slot_rows + lr;
    if (tj * BN + cq < p.rows_b) store_vals<T>(p, gi, tj * BN + cq, v, 4);
  }
}

template <typename T, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tcgen05_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b, const TcParams p) {
  using L = TcLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* red_full = acc_full + 1;  // push split-K: the peers' rows have arrived
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_full + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] last split

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const bool push = L::kPush && p.splits > 1;
  int ti, tj;
  tile_coords(tile, p.tiles_i, p.tiles_j, ti, tj);
  // K blocks are spread evenly over the splits (the plan keeps >= 1 per split).
  const int kb0 = static_cast<int>(static_cast<int64_t>(split) * p.kblocks / p.splits);
  const int nkb = static_cast<int>(static_cast<int64_t>(split + 1) * p.kblocks / p.splits) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(red_full, 1);
    if (push)  // the peers' rows of this rank: (S - 1) senders x its rows x BN floats
      mbar_arrive_expect_tx(red_full, static_cast<uint32_t>((p.splits - 1) *
                                                            push_my_rows(p.epilogue, p.splits, split) * BN * 4));
    flags[0] = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (push) cluster_arrive();  // this rank's receive barrier is ready for its peers
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // Weight tiles of the first stages do not depend on the previous kernel:
      // stream them while that kernel finishes, then wait for its outputs.
      const int pre = (p.const_a || p.const_b) ? min(STAGES, nkb) : 0;
      for (int it = 0; it < pre; ++it) {
        uint8_t* sa = smem + it * L::kStageBytes;
        mbar_arrive_expect_tx(&full[it], L::kStageBytes);
        if (p.const_a) tma_load_2d(sa, &tmap_a, (kb0 + it) * kBK, ti * kBM, &full[it]);
        else load_b_block<BN>(sa + L::kABytes, &tmap_b, kb0 + it, tj, p.b_mn, &full[it]);
      }
      pdl_wait();
      pdl_trigger();
      int issued = pre;
      for (int it = 0; it < nkb; ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        uint8_t* sa = smem + s * L::kStageBytes;
        if (it < pre) {  // stage armed above: add the dependent operand
          if (p.const_a) load_b_block<BN>(sa + L::kABytes, &tmap_b, kb0 + it, tj, p.b_mn, &full[s]);
          else tma_load_2d(sa, &tmap_a, (kb0 + it) * kBK, ti * kBM, &full[s]);
          continue;
        }
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        if (flags[0]) break;
        mbar_arrive_expect_tx(&full[s], L::kStageBytes);
        tma_load_2d(sa, &tmap_a, (kb0 + it) * kBK, ti * kBM, &full[s]);
        load_b_block<BN>(sa + L::kABytes, &tmap_b, kb0 + it, tj, p.b_mn, &full[s]);
        issued = it + 1;
      }
      // No bulk copy may still be writing shared memory when the CTA exits.
      for (int it = max(0, issued - STAGES); it < issued; ++it)
        mbar_wait(&full[it % STAGES], (it / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc =
          umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, kBM, BN) | (p.b_mn ? (1u << 16) : 0u);
      for (int it = 0; it < nkb; ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full[s], ph)) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes);
        const uint64_t adesc = umma_desc_sw128(a_addr);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16(tmem_base, adesc + 2 * kk, b_block_desc(a_addr + L::kABytes, kk, p.b_mn), idesc,
                   (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(acc_full);
    }
  } else {
    if (push) tile_push_partial<T, BN, STAGES>(p, smem, tmem_base, acc_full, red_full, flags, split, warp, lane);
    else tile_epilogue_warps<T, BN>(p, smem, tmem_base, acc_full, flags, ti, tj, warp, lane);
  }
  if (push && warp < 2) cluster_wait();  // pairs this thread's arrival at kernel start
  tc_fence_before();
  __syncthreads();
  if (push) tile_push_reduce<T, BN, STAGES>(p, smem, red_full, ti, tj, split);
  else if (p.splits > 1) tile_cluster_reduce<T, BN>(p, smem, ti, tj, split);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---- implicit-GEMM convolution on tcgen05 ---------------------------------------
// D[m, oc] = sum_k patch[m, k] * W[oc, k] with m = (image, output pixel) and
// k = (channel, ky, kx), the weight's own [OC, C, KH, KW] order. No patch
// matrix is written: eight gather warps build each 128-pixel x 64-k A tile in
// shared memory straight from the NCHW input (thread = one pixel row and one
// half of the block's k values; the (channel, ky, kx) of each k comes from a
// per-block table, so the 32 loads carry no branches and are all in flight at
// once; zero outside the image and past K), 128B-swizzled like a TMA box,
// while warp 0 streams the K-major weight tiles by TMA. MMA, split-K and the
// NCHW epilogue (warps 2-5) are the GEMM kernel's.
constexpr int kConvThreads = 320;
constexpr int kConvGatherThreads = 256;

template <typename T, int BN, int STAGES>
__global__ void __launch_bounds__(kConvThreads, 1)
    tcgen05_conv_kernel(const __grid_constant__ CUtensorMap tmap_b, const TcParams p, const T* __restrict__ x,
                        const ConvGeom g) {
  using L = TcLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);  // weight tile landed (TMA)
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* red_full = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_full + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [STAGES] patch tile written: after the GEMM layout's barriers, slot and flags
  uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset + (2 * STAGES + 2) * 8 + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const bool push = L::kPush && p.splits > 1;
  int ti, tj;
  tile_coords(tile, p.tiles_i, p.tiles_j, ti, tj);
  const int kb0 = static_cast<int>(static_cast<int64_t>(split) * p.kblocks / p.splits);
  const int nkb = static_cast<int>(static_cast<int64_t>(split + 1) * p.kblocks / p.splits) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&a_full[s], 8);  // one arrive per gather warp
    }
    mbar_init(acc_full, 1);
    mbar_init(red_full, 1);
    if (push)
      mbar_arrive_expect_tx(red_full, static_cast<uint32_t>((p.splits - 1) *
                                                            push_my_rows(p.epilogue, p.splits, split) * BN * 4));
    flags[0] = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmap_b);
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (push) cluster_arrive();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // the weights do not depend on the previous kernel: their first tiles load before the wait
      const int pre = min(STAGES, nkb);
      for (int it = 0; it < pre; ++it) {
        mbar_arrive_expect_tx(&full[it], L::kBBytes);
        tma_load_2d(smem + it * L::kStageBytes + L::kABytes, &tmap_b, (kb0 + it) * kBK, tj * BN, &full[it]);
      }
      pdl_wait();
      pdl_trigger();
      int issued = pre;
      for (int it = pre; it < nkb; ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1) || flags[0]) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], L::kBBytes);
        tma_load_2d(smem + s * L::kStageBytes + L::kABytes, &tmap_b, (kb0 + it) * kBK, tj * BN, &full[s]);
        issued = it + 1;
      }
      for (int it = max(0, issued - STAGES); it < issued; ++it) mbar_wait(&full[it % STAGES], (it / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, kBM, BN);
      for (int it = 0; it < nkb; ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full[s], ph) || !mbar_wait(&a_full[s], ph)) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes);
        const uint64_t adesc = umma_desc_sw128(a_addr);
        const uint64_t bdesc = umma_desc_sw128(a_addr + L::kABytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16(tmem_base, adesc + 2 * kk, bdesc + 2 * kk, idesc, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(acc_full);
    }
  } else {
    // gather warps 2-9: thread = one output pixel (A row) and one half of the k block
    const int gtid = threadIdx.x - 64;
    const int row = gtid & (kBM - 1), khalf = gtid >> 7;
    const int64_t m = static_cast<int64_t>(ti) * kBM + row;
    const int ohw = g.oh * g.ow, khw = g.kh * g.kw, hw = g.h * g.w;
    const bool live = m < p.rows_a;
    const int img = live ? static_cast<int>(m / ohw) : 0;
    const int pix = live ? static_cast<int>(m - static_cast<int64_t>(img) * ohw) : 0;
    const int iy0 = (pix / g.ow) * g.sh - g.ph, ix0 = (pix % g.ow) * g.sw - g.pw;
    const unsigned short* xb = reinterpret_cast<const unsigned short*>(x) + static_cast<int64_t>(img) * g.c * hw;
    const int pbase = iy0 * g.w + ix0;  // + (c*H + ky)*W + kx = the element's offset in the image
    const int kdim = g.c * khw;
    int2* ktable = reinterpret_cast<int2*>(a_full + STAGES);                  // [2][kBK]
    volatile int* votes = reinterpret_cast<volatile int*>(ktable + 2 * kBK);  // [2][8]
    pdl_wait();  // the input is the previous kernel's output
    for (int it = 0; it < nkb; ++it) {
      const int s = it % STAGES;
      const bool w = mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1);
      const int abort_seen = __shfl_sync(0xffffffffu, flags[0], 0);
      const bool warp_ok = __all_sync(0xffffffffu, w) && !abort_seen;
      // the (channel, ky, kx) of the block's 64 k values, shared by every pixel
      // row. Table and votes are double-buffered, so one barrier per block
      // suffices; every gather warp reaches it on every block (the waits above
      // are bounded) and the votes make the abort decision the same in all.
      int2* tbl = ktable + (it & 1) * kBK;
      if (gtid < kBK) {
        const int k = (kb0 + it) * kBK + gtid;
        const int c = k / khw, r = k - c * khw, ky = r / g.kw, kx = r - ky * g.kw;
        tbl[gtid] = k < kdim ? make_int2((c * g.h + ky) * g.w + kx, (ky << 16) | kx) : make_int2(-1, 0);
      }
      if (lane == 0) votes[(it & 1) * 8 + (warp - 2)] = warp_ok ? 1 : 0;
      asm volatile("bar.sync 2, %0;" ::"n"(kConvGatherThreads) : "memory");
      volatile const int* vt = votes + (it & 1) * 8;
      bool all_ok = true;
#pragma unroll
      for (int i = 0; i < 8; ++i) all_ok = all_ok && vt[i] != 0;
      if (!all_ok) {
        if (lane == 0) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
        }
        break;
      }
      uint32_t v[kBK / 4];
#pragma unroll
      for (int e = 0; e < kBK / 2; e += 2) {
        uint32_t pair = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int2 t = tbl[khalf * (kBK / 2) + e + h];
          const int iy = iy0 + (t.y >> 16), ix = ix0 + (t.y & 0xffff);
          const bool ok = live && t.x >= 0 && static_cast<unsigned>(iy) < static_cast<unsigned>(g.h) &&
                          static_cast<unsigned>(ix) < static_cast<unsigned>(g.w);
          // unconditional load (element 0 of the image when outside it), then a
          // select: no branch between the loads, so all are in flight at once
          const uint32_t raw = __ldg(xb + (ok ? pbase + t.x : 0));
          pair |= (ok ? raw : 0u) << (16 * h);
        }
        v[e >> 1] = pair;
      }
      uint8_t* a_tile = smem + s * L::kStageBytes + row * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int chunk = khalf * 4 + q;
        *reinterpret_cast<uint4*>(a_tile + ((chunk ^ (row & 7)) << 4)) =
            make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
      fence_proxy_async_smem();  // read by the tensor core (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
    }
    if (warp < 6) {  // the epilogue runs on warps 2-5 (one TMEM lane quarter each)
      if (push) tile_push_partial<T, BN, STAGES>(p, smem, tmem_base, acc_full, red_full, flags, split, warp, lane);
      else tile_epilogue_warps<T, BN>(p, smem, tmem_base, acc_full, flags, ti, tj, warp, lane);
    }
  }
  if (push && (warp < 2 || warp >= 6)) cluster_wait();  // the threads that push nothing
  tc_fence_before();
  __syncthreads();
  if (push) tile_push_reduce<T, BN, STAGES, kConvThreads>(p, smem, red_full, ti, tj, split);
  else if (p.splits > 1) tile_cluster_reduce<T, BN, kConvThreads>(p, smem, ti, tj, split);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---- fp32 GEMM on tcgen05 through a three-term bf16 split -----------------------
// fp32 operands stream in by TMA unchanged (128B-swizzled boxes of 32 floats).
// Converter warps split every element into three bf16 terms, x = h + m + l with
// h = bf16(x), m = bf16(x - h), l = bf16(x - h - m) (both differences exact in
// fp32), and write them as the operand tiles of f16-kind MMAs. Each 64-wide K
// block accumulates the six products whose order is at most 2^-16 below x*y
// (h*l, l*h, m*m, h*m, m*h, h*h) into a fresh tensor-memory buffer; the same
// warps then add that block partial into fp32 registers with round-to-nearest
// adds. The tensor core's own accumulation loses a little on every MMA it adds
// into a running sum (the error grows with the number of MMAs per sum), so
// bounding each hardware sum to one K block and promoting block sums to
// registers keeps the result at the accuracy of an fp32 FFMA GEMM. Dropped split
// terms are near 2^-26 of each product. Non-finite inputs keep h, with m = l = 0.
//
// 320 threads: warp 0 TMA producer, warp 1 TMEM owner and MMA issuer, warps 2-9
// converters, promoters and epilogue (warp w reads TMEM lanes 32*(w%4).. and
// column half (w-2)/4 of each block). Rings: raw (TMA -> converters), converted
// (converters -> MMA) and the two block-partial buffers in tensor memory
// (MMA -> promoters), every wait bounded. Split-K partials are reduced over the
// cluster like the bf16 kernel's, storing float32.
constexpr int kSplitTerms = 3;
constexpr int kF32SplitThreads = 320;
constexpr int kF32SplitWorkers = 256;  // warps 2-9

template <int BN, int RS, int CS>
struct F32x3Layout {
  static constexpr int kRawStageBytes = (kBM + BN) * 256;                 // fp32 [A | B] of one K block
  static constexpr int kCvStageBytes = (kBM + BN) * 128 * kSplitTerms;   // bf16 [A h|m|l | B h|m|l]
  static constexpr int kCvOff = RS * kRawStageBytes;
  static constexpr int kBarOffset = kCvOff + CS * kCvStageBytes;
  // raw_full[RS], raw_empty[RS], cv_full[CS], cv_empty[CS], acc_full[2], acc_empty[2], mma_done
  static constexpr int kBytes = kBarOffset + (2 * RS + 2 * CS + 5) * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // two block-partial buffers
  static_assert(kBM * (BN + 4) * 4 <= kBarOffset, "split-K staging must fit the rings");
  static_assert(kBytes <= 232448, "shared memory per CTA");
};

// Splits 4 floats into three bf16 terms, stored as 8 bytes in each plane
// (planes `plane` bytes apart).
__device__ __forceinline__ void split_bf16x4(const float4 v, uint8_t* dst, int plane) {
  const float x[4] = {v.x, v.y, v.z, v.w};
  uint32_t w[3][2];
#pragma unroll
  for (int e = 0; e < 4; e += 2) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x[e], x[e + 1]);
    const float2 hf = __bfloat1622float2(h);
    const bool fin0 = fabsf(hf.x) < __int_as_float(0x7f800000), fin1 = fabsf(hf.y) < __int_as_float(0x7f800000);
    const float r0 = fin0 ? x[e] - hf.x : 0.f, r1 = fin1 ? x[e + 1] - hf.y : 0.f;
    const __nv_bfloat162 m = __floats2bfloat162_rn(r0, r1);
    const float2 mf = __bfloat1622float2(m);
    const __nv_bfloat162 l = __floats2bfloat162_rn(r0 - mf.x, r1 - mf.y);
    w[0][e / 2] = *reinterpret_cast<const uint32_t*>(&h);
    w[1][e / 2] = *reinterpret_cast<const uint32_t*>(&m);
    w[2][e / 2] = *reinterpret_cast<const uint32_t*>(&l);
  }
#pragma unroll
  for (int t = 0; t < 3; ++t) *reinterpret_cast<uint2*>(dst + t * plane) = make_uint2(w[t][0], w[t][1]);
}

// Converts one operand block of `rows` rows x 64 K (or, MN-major, 64 K rows per
// 64-column panel) from its raw fp32 boxes to 128B-swizzled bf16 planes
// (`plane` bytes apart). Raw boxes come in groups of G rows: group g, K half h
// at (2g + h) * G * 128 bytes, row r % G at 128 bytes per row, 16-byte chunks
// XOR-swizzled by r % 8. Converted row r sits at r * 128 with chunks swizzled
// the same way. One task is one raw chunk (4 floats): 8 consecutive threads read
// one 128-byte box row and 16 consecutive threads write one 128-byte bf16 row,
// both conflict-free.
__device__ __forceinline__ void split_block(const uint8_t* raw, int G, int rows, uint8_t* cv, int plane, int tid) {
#pragma unroll 2
  for (int t = tid; t < rows * 16; t += kF32SplitWorkers) {
    const int r = t >> 4, h = (t >> 3) & 1, qc = t & 7, sw = r & 7;
    const int g = r / G, rg = r - g * G;
    const float4 v = *reinterpret_cast<const float4*>(raw + (2 * g + h) * G * 128 + rg * 128 + ((qc ^ sw) << 4));
    const int off = r * 128 + (((h * 4 + (qc >> 1)) ^ sw) << 4) + (qc & 1) * 8;
    split_bf16x4(v, cv + off, plane);
  }
}

// Adds n (16 or 32) tensor-memory columns of this thread's lane into acc.
template <int N>
__device__ __forceinline__ void tmem_add_cols(uint32_t taddr, float* acc) {
  if constexpr (N == 16) {
    uint32_t r[16];
    tmem_ld_32x32b_x16(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] += __uint_as_float(r[i]);
  } else {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] += __uint_as_float(r[i]);
  }
}

template <int BN, int RS, int CS>
__global__ void __launch_bounds__(kF32SplitThreads, 1)
    tcgen05_gemm_f32x3_kernel(const __grid_constant__ CUtensorMap tmap_a,
                              const __grid_constant__ CUtensorMap tmap_b, const TcParams p) {
  using L = F32x3Layout<BN, RS, CS>;
  constexpr int HALF = BN / 2;                 // columns per promoter thread
  constexpr int CH = HALF < 32 ? HALF : 32;    // columns per TMEM load
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* cv_full = raw_empty + RS;
  uint64_t* cv_empty = cv_full + CS;
  uint64_t* acc_full = cv_empty + CS;   // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  int ti, tj;
  tile_coords(tile, p.tiles_i, p.tiles_j, ti, tj);
  const int kb0 = static_cast<int>(static_cast<int64_t>(split) * p.kblocks / p.splits);
  const int nkb = static_cast<int>(static_cast<int64_t>(split + 1) * p.kblocks / p.splits) - kb0;

  if (threadIdx.x == 0) {
    mbar_init(mma_done, 1);
    for (int s = 0; s < RS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 8);  // one arrive per converter warp
    }
    for (int s = 0; s < CS; ++s) {
      mbar_init(&cv_full[s], 8);
      mbar_init(&cv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrive per promoter warp
    }
    flags[0] = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      pdl_trigger();
      int issued = 0;
      for (int it = 0; it < nkb; ++it) {
        const int s = it % RS;
        if (!mbar_wait(&raw_empty[s], ((it / RS) & 1) ^ 1)) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        if (flags[0]) break;
        uint8_t* ra = smem + s * L::kRawStageBytes;
        uint8_t* rb = ra + kBM * 256;
        const int k0 = (kb0 + it) * kBK;
        mbar_arrive_expect_tx(&raw_full[s], L::kRawStageBytes);
        tma_load_2d(ra, &tmap_a, k0, ti * kBM, &raw_full[s]);
        tma_load_2d(ra + kBM * 128, &tmap_a, k0 + 32, ti * kBM, &raw_full[s]);
        if (p.b_mn) {
#pragma unroll
          for (int q = 0; q < 2 * (BN / 64); ++q)
            tma_load_2d(rb + q * 64 * 128, &tmap_b, tj * BN + q * 32, k0, &raw_full[s]);
        } else {
          tma_load_2d(rb, &tmap_b, k0, tj * BN, &raw_full[s]);
          tma_load_2d(rb + BN * 128, &tmap_b, k0 + 32, tj * BN, &raw_full[s]);
        }
        issued = it + 1;
      }
      // No bulk copy may still be writing shared memory when the CTA exits.
      for (int it = max(0, issued - RS); it < issued; ++it) mbar_wait(&raw_full[it % RS], (it / RS) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(true, kBM, BN) | (p.b_mn ? (1u << 16) : 0u);
      int done = 0;
      for (int it = 0; it < nkb; ++it) {
        const int s = it % CS, b = it & 1;
        if (!mbar_wait(&cv_full[s], (it / CS) & 1) || !mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1) || flags[0]) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_h = smem_u32(smem + L::kCvOff + s * L::kCvStageBytes);
        const uint32_t a_m = a_h + kBM * 128, a_l = a_m + kBM * 128;
        const uint32_t b_h = a_h + kSplitTerms * kBM * 128, b_m = b_h + BN * 128, b_l = b_m + BN * 128;
        const uint32_t acc = tmem_base + static_cast<uint32_t>(b * BN);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t ah = umma_desc_sw128(a_h) + 2 * kk, am = umma_desc_sw128(a_m) + 2 * kk,
                         al = umma_desc_sw128(a_l) + 2 * kk;
          const uint64_t bh = b_block_desc(b_h, kk, p.b_mn), bm = b_block_desc(b_m, kk, p.b_mn),
                         bl = b_block_desc(b_l, kk, p.b_mn);
          umma_f16(acc, ah, bl, idesc, kk > 0 ? 1u : 0u);  // a fresh sum per K block
          umma_f16(acc, al, bh, idesc, 1u);
          umma_f16(acc, am, bm, idesc, 1u);
          umma_f16(acc, ah, bm, idesc, 1u);
          umma_f16(acc, am, bh, idesc, 1u);
          umma_f16(acc, ah, bh, idesc, 1u);
        }
        umma_commit(&cv_empty[s]);
        umma_commit(&acc_full[b]);
        done = it + 1;
      }
      if (done < nkb) {  // aborted: release promoters waiting on a block that never comes
        umma_commit(&acc_full[0]);
        umma_commit(&acc_full[1]);
      }
      // every issued MMA has finished before the CTA releases tensor memory
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else {
    // warps 2-9: convert block it, then promote block it-1 (its MMAs overlap the
    // conversion of block it); the last block is promoted after the loop
    const int tid = threadIdx.x - 64;
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(half * HALF);
    float accum[HALF];
#pragma unroll
    for (int i = 0; i < HALF; ++i) accum[i] = 0.f;
    bool ok = true;
    auto promote = [&](int j) -> bool {
      const int b = j & 1;
      const bool w = mbar_wait(&acc_full[b], (j >> 1) & 1);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HALF; c += CH) tmem_add_cols<CH>(lane_base + static_cast<uint32_t>(b * BN + c), accum + c);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      return true;
    };
    for (int it = 0; it < nkb && ok; ++it) {
      const int rs = it % RS, cs = it % CS;
      bool w = mbar_wait(&raw_full[rs], (it / RS) & 1);
      w = w && mbar_wait(&cv_empty[cs], ((it / CS) & 1) ^ 1);
      const int abort_seen = __shfl_sync(0xffffffffu, flags[0], 0);
      if (!__all_sync(0xffffffffu, w) || abort_seen) {
        ok = false;
        break;
      }
      const uint8_t* ra = smem + rs * L::kRawStageBytes;
      uint8_t* cv = smem + L::kCvOff + cs * L::kCvStageBytes;
      split_block(ra, kBM, kBM, cv, kBM * 128, tid);
      split_block(ra + kBM * 256, p.b_mn ? 64 : BN, BN, cv + kSplitTerms * kBM * 128, BN * 128, tid);
      fence_proxy_async_smem();  // the bf16 tiles are read by the tensor core (async proxy)
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[rs]);
        mbar_arrive(&cv_full[cs]);
      }
      if (it > 0) ok = promote(it - 1);
    }
    if (ok && nkb > 0) ok = promote(nkb - 1);
    if (!ok) {
      if (lane == 0) {
        set_device_error(p.err, kDevErrGemmTimeout);
        flags[0] = 1;
      }
    }
    // named barrier over the 8 epilogue warps: every one sees the same abort flag
    asm volatile("bar.sync 1, %0;" ::"n"(kF32SplitWorkers) : "memory");
    const bool aborted = flags[0] != 0;
    const int64_t gi = static_cast<int64_t>(ti) * kBM + row;
    const int jc = tj * BN + half * HALF;
    if (p.splits == 1) {
      if (!aborted) {
#pragma unroll
        for (int c = 0; c < HALF; c += CH) {
          float v[CH];  // a copy: accum stays in registers (constant indices only)
#pragma unroll
          for (int i = 0; i < CH; ++i) v[i] = accum[c + i];
          if (jc + c < p.rows_b) store_vals<__nv_bfloat16>(p, gi, jc + c, v, CH);
        }
      }
    } else {
      float* red = reinterpret_cast<float*>(smem);  // the idle raw ring: [128][BN + 4]
#pragma unroll
      for (int c = 0; c < HALF; c += 4)
        *reinterpret_cast<float4*>(red + row * (BN + 4) + half * HALF + c) =
            aborted ? make_float4(0.f, 0.f, 0.f, 0.f)
                    : make_float4(accum[c], accum[c + 1], accum[c + 2], accum[c + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (p.splits > 1) tile_cluster_reduce<__nv_bfloat16, BN, kF32SplitThreads>(p, smem, ti, tj, split);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---- persistent tcgen05 GEMM (prefill-sized problems) --------------------------
// One CTA per SM walks tiles blockIdx.x, +gridDim.x, ... (grouped raster). The
// accumulator is double-buffered in tensor memory (2 x 256 columns = all 512):
// while the epilogue warps drain tile n from one buffer, the MMA warp already
// accumulates tile n+1 into the other, and the producer streams its operands,
// so tile epilogues no longer stall the tensor pipe. acc_full[b] (MMA ->
// epilogue, tcgen05.commit) and acc_empty[b] (4 epilogue warps -> MMA) hand the
// buffers over; the operand ring runs across tile boundaries.
template <int STAGES>
struct PersistentLayout {
  static constexpr int BN = 256;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBytes = kBarOffset + (2 * STAGES + 4) * 8 + 16 + 1024;
};

template <typename T, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tcgen05_gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                   const __grid_constant__ CUtensorMap tmap_b, const TcParams p) {
  using L = PersistentLayout<STAGES>;
  constexpr int BN = L::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.tiles_i * p.tiles_j;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrive per epilogue warp
    }
    flags[0] = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      pdl_trigger();
      int it = 0;
      bool stop = false;
      for (int tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x) {
        int ti, tj;
        tile_coords(tile, p.tiles_i, p.tiles_j, ti, tj);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            set_device_error(p.err, kDevErrGemmTimeout);
            flags[0] = 1;
          }
          if (flags[0]) {
            stop = true;
            break;
          }
          uint8_t* sa = smem + s * L::kStageBytes;
          mbar_arrive_expect_tx(&full[s], L::kStageBytes);
          tma_load_2d(sa, &tmap_a, kb * kBK, ti * kBM, &full[s]);
          load_b_block<BN>(sa + L::kABytes, &tmap_b, kb, tj, p.b_mn, &full[s]);
          ++it;
        }
      }
      // No bulk copy may still be writing shared memory when the CTA exits.
      for (int j = max(0, it - STAGES); j < it; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc =
          umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, kBM, BN) | (p.b_mn ? (1u << 16) : 0u);
      int it = 0, lt = 0;
      bool stop = false;
      for (int tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1) || flags[0]) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph)) {
            set_device_error(p.err, kDevErrGemmTimeout);
            flags[0] = 1;
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes);
          const uint64_t adesc = umma_desc_sw128(a_addr);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(acc, adesc + 2 * kk, b_block_desc(a_addr + L::kABytes, kk, p.b_mn), idesc,
                     (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          ++it;
        }
        umma_commit(&acc_full[buf]);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
      const int buf = lt & 1;
      if (!mbar_wait(&acc_full[buf], (lt >> 1) & 1)) {
        set_device_error(p.err, kDevErrGemmTimeout);
        flags[0] = 1;
      }
      tc_fence_after();
      epilogue_bar();  // every epilogue warp sees the same abort flag
      if (flags[0]) break;
      int ti, tj;
      tile_coords(tile, p.tiles_i, p.tiles_j, ti, tj);
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
      epilogue_tile<T, BN>(p, tbase, static_cast<int64_t>(ti) * kBM + row, tj * BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ---- stream-K GEMM for decode-sized (swap-AB) problems ----------------------------
// The (tile, K block) work units of a skinny GEMM are split evenly over P CTAs
// (P = every resident slot of the GPU, two per SM), so every SM streams the same
// number of weight bytes whatever the tile count: a CTA's contiguous unit range
// may end inside one tile and start inside another. A CTA that covers a whole
// tile stores it directly; a CTA holding part of a tile writes its fp32 partial
// to the workspace and counts itself in; the last arrival sums the partials of
// all contributors in CTA order (a fixed order, so the result is deterministic)
// and stores the tile. No CTA waits for another, and no thread-block clusters
// constrain where CTAs may run, so the next kernel's CTAs (programmatic
// dependent launch) start on every SM as soon as this kernel's leave it.
// Accumulators are double-buffered in TMEM: the MMA warp starts a CTA's next
// segment while the epilogue drains the previous one.
template <int BN, int STAGES>
struct StreamKLayout {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kXchOffset = (kBarOffset + (2 * STAGES + 4) * 8 + 16 + 127) / 128 * 128;
  static constexpr int kXchFloats = 64 * (BN + 1);  // SwiGLU: up rows handed to the gate rows
  static constexpr int kBytes = kXchOffset + kXchFloats * 4 + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzle atoms need 1 KiB alignment");
};

// First work unit of CTA c when U units are split over P CTAs.
__device__ __forceinline__ int64_t sk_begin(int64_t c, int64_t units, int64_t ctas) { return c * units / ctas; }
// The CTA whose unit range holds unit u.
__device__ __forceinline__ int sk_owner(int64_t u, int64_t units, int64_t ctas) {
  int64_t c = u * ctas / units;
  while (c + 1 < ctas && sk_begin(c + 1, units, ctas) <= u) ++c;
  while (c > 0 && sk_begin(c, units, ctas) > u) --c;
  return static_cast<int>(c);
}

template <typename T, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tcgen05_gemm_streamk_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                const __grid_constant__ CUtensorMap tmap_b, const TcParams p) {
  using L = StreamKLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] last arrival
  float* xch = reinterpret_cast<float*>(smem + L::kXchOffset);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t units = static_cast<int64_t>(p.tiles_i) * p.tiles_j * p.kblocks;
  const int64_t ctas = gridDim.x;
  const int c = blockIdx.x;
  const int64_t u_begin = sk_begin(c, units, ctas), u_end = sk_begin(c + 1, units, ctas);
  const int first_tile = static_cast<int>(u_begin / p.kblocks);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    flags[0] = 0;
    flags[1] = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // the weight tiles of the first stages do not depend on the previous kernel
      int issued = 0;
      const int pre = p.const_a ? static_cast<int>((u_end - u_begin < STAGES ? u_end - u_begin : STAGES)) : 0;
      for (int it = 0; it < pre; ++it) {
        const int64_t u = u_begin + it;
        int ti, tj;
        tile_coords(static_cast<int>(u / p.kblocks), p.tiles_i, p.tiles_j, ti, tj);
        mbar_arrive_expect_tx(&full[it], L::kStageBytes);
        tma_load_2d(smem + it * L::kStageBytes, &tmap_a, static_cast<int>(u % p.kblocks) * kBK, ti * kBM, &full[it]);
      }
      pdl_wait();
      pdl_trigger();
      for (int64_t u = u_begin; u < u_end; ++u) {
        const int it = static_cast<int>(u - u_begin);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        int ti, tj;
        tile_coords(static_cast<int>(u / p.kblocks), p.tiles_i, p.tiles_j, ti, tj);
        const int kx = static_cast<int>(u % p.kblocks) * kBK;
        uint8_t* sa = smem + s * L::kStageBytes;
        if (it < pre) {  // armed above: add the activations
          tma_load_2d(sa + L::kABytes, &tmap_b, kx, tj * BN, &full[s]);
          issued = it + 1;
          continue;
        }
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
        }
        if (flags[0]) break;
        mbar_arrive_expect_tx(&full[s], L::kStageBytes);
        tma_load_2d(sa, &tmap_a, kx, ti * kBM, &full[s]);
        tma_load_2d(sa + L::kABytes, &tmap_b, kx, tj * BN, &full[s]);
        issued = it + 1;
      }
      // No bulk copy may still be writing shared memory when the CTA exits.
      for (int it = max(0, issued - STAGES); it < issued; ++it) mbar_wait(&full[it % STAGES], (it / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, kBM, BN);
      int64_t u = u_begin;
      for (int ls = 0; u < u_end && !flags[0]; ++ls) {
        const int buf = ls & 1;
        const int64_t seg_end = u_end < (u / p.kblocks + 1) * p.kblocks ? u_end : (u / p.kblocks + 1) * p.kblocks;
        if (!mbar_wait(&acc_empty[buf], ((ls >> 1) & 1) ^ 1) || flags[0]) {
          set_device_error(p.err, kDevErrGemmTimeout);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + static_cast<uint32_t>(buf * BN);
        bool first = true;
        for (; u < seg_end; ++u) {
          const int it = static_cast<int>(u - u_begin);
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1)) {
            set_device_error(p.err, kDevErrGemmTimeout);
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes);
          const uint64_t adesc = umma_desc_sw128(a_addr);
          const uint64_t bdesc = umma_desc_sw128(a_addr + L::kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (!first || kk > 0) ? 1u : 0u);
          first = false;
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[buf]);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane = weight row of the tile
    int64_t u = u_begin;
    for (int ls = 0; u < u_end; ++ls) {
      const int buf = ls & 1;
      const int tile = static_cast<int>(u / p.kblocks);
      const int64_t tile_u0 = static_cast<int64_t>(tile) * p.kblocks;
      const int64_t seg_end = u_end < tile_u0 + p.kblocks ? u_end : tile_u0 + p.kblocks;
      const bool whole = u == tile_u0 && seg_end == tile_u0 + p.kblocks;
      u = seg_end;
      if (!mbar_wait(&acc_full[buf], (ls >> 1) & 1)) {
        set_device_error(p.err, kDevErrGemmTimeout);
        flags[0] = 1;
      }
      tc_fence_after();
      epilogue_bar();  // every epilogue warp sees the same abort flag
      if (flags[0]) break;
      float v[BN];
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
#pragma unroll
      for (int cc = 0; cc < BN; cc += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + cc, r);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 32; ++k) v[cc + k] = __uint_as_float(r[k]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);  // the MMA warp may reuse this buffer
      if (!whole) {
        // partial tile: publish it, count in, and the last contributor sums all of them
        const int slot = tile == first_tile ? 0 : 1;
        float* mine = p.sk_part + ((static_cast<int64_t>(c) * 2 + slot) * kBM + row) * BN;
#pragma unroll
        for (int cc = 0; cc < BN; cc += 4)
          __stcg(reinterpret_cast<float4*>(mine + cc), make_float4(v[cc], v[cc + 1], v[cc + 2], v[cc + 3]));
        __threadfence();
        epilogue_bar();
        const int c_first = sk_owner(tile_u0, units, ctas);
        const int c_last = sk_owner(tile_u0 + p.kblocks - 1, units, ctas);
        if (row == 0) flags[1] = atomicAdd(p.sk_count + tile, 1) == c_last - c_first;
        epilogue_bar();
        const bool last = flags[1] != 0;
        if (!last) continue;
        __threadfence();
#pragma unroll
        for (int k = 0; k < BN; ++k) v[k] = 0.f;
        for (int cc2 = c_first; cc2 <= c_last; ++cc2) {  // CTA order: a fixed summation order
          const int ctile = static_cast<int>(sk_begin(cc2, units, ctas) / p.kblocks);
          const float* src = p.sk_part + ((static_cast<int64_t>(cc2) * 2 + (tile == ctile ? 0 : 1)) * kBM + row) * BN;
#pragma unroll
          for (int cc = 0; cc < BN; cc += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(src + cc));
            v[cc] += x.x;
            v[cc + 1] += x.y;
            v[cc + 2] += x.z;
            v[cc + 3] += x.w;
          }
        }
        if (row == 0) p.sk_count[tile] = 0;  // ready for the next call (graph replays included)
      }
      // the finished tile
      int ti, tj;
      tile_coords(tile, p.tiles_i, p.tiles_j, ti, tj);
      const int64_t gi = static_cast<int64_t>(ti) * kBM + row;
      if (p.epilogue == kEpiGluT) {
        if (quarter >= 2) {
#pragma unroll
          for (int k = 0; k < BN; ++k) xch[(row - 64) * (BN + 1) + k] = v[k];
        }
        epilogue_bar();
        if (quarter < 2) {
          const float* up = xch + row * (BN + 1);
          store_glu_t<T>(p, ti, row, tj * BN, v, up, BN);
        }
        epilogue_bar();
      } else {
#pragma unroll
        for (int cc = 0; cc < BN; cc += 32)
          if (tj * BN + cc < p.rows_b) store_vals<T>(p, gi, tj * BN + cc, v + cc, 32);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---- SIMT fallback -----------------------------------------------------------
constexpr int kSimtTile = 64;
constexpr int kSimtK = 16;

template <typename T, bool kBKMajor>
__global__ void __launch_bounds__(256)
    gemm_simt_kernel(const T* __restrict__ a, const T* __restrict__ b, const T* __restrict__ bias,
                     T* __restrict__ out, int64_t m, int64_t n, int64_t k) {
  DLI_PDL_ENTRY();
  __shared__ float as[kSimtK][kSimtTile + 4];
  __shared__ float bs[kSimtK][kSimtTile + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kSimtTile;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kSimtTile;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < k; k0 += kSimtK) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = tid + e * 256;
      const int r = idx >> 4, c = idx & 15;
      as[c][r] = (m0 + r < m && k0 + c < k) ? to_f32(a[(m0 + r) * k + k0 + c]) : 0.f;
      if constexpr (kBKMajor) {
        bs[c][r] = (n0 + r < n && k0 + c < k) ? to_f32(b[(n0 + r) * k + k0 + c]) : 0.f;
      } else {
        const int kk = idx >> 6, nn = idx & 63;
        bs[kk][nn] = (k0 + kk < k && n0 + nn < n) ? to_f32(b[(k0 + kk) * n + n0 + nn]) : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSimtK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = as[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty * 4 + i;
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = n0 + tx * 4 + j;
      if (c < n) out[r * n + c] = from_f32<T>(acc[i][j] + (bias ? to_f32(bias[c]) : 0.f));
    }
  }
}

// ---- exact fp32 GEMM on CUDA cores, split-K over a thread-block cluster ----------
// out[M,N] = A[M,K] . B + bias with B as [N,K] (linear) or [K,N] (matmul), fp32
// FFMA in the reference's accumulation precision (its tl.dot runs fp32 as TF32,
// 1e-3 relative; this kernel is exact fp32). CTA tile 64 x 128, 256 threads of
// 4 x 8 outputs, K in 16-deep slices double-buffered in shared memory (16-byte
// global loads). Skinny problems (decode-sized M) split K over S <= 8 CTAs that
// form one thread-block cluster: each stages its fp32 partial tile in its own
// shared memory, and after a cluster barrier CTA r sums rows r*64/S.. of all S
// partials in rank order through distributed shared memory (deterministic, no
// workspace, no second launch).
constexpr int kF32BM = 64, kF32BN = 128, kF32BK = 16, kF32Threads = 256;
constexpr int kF32AStride = kF32BM + 4, kF32BStride = kF32BN + 4;
constexpr int kF32StageFloats = kF32BK * (kF32AStride + kF32BStride);
constexpr int kF32RedStride = kF32BN + 4;
constexpr int kF32SmemBytes =
    (2 * kF32StageFloats > kF32BM * kF32RedStride ? 2 * kF32StageFloats : kF32BM * kF32RedStride) * 4;

struct F32GemmArgs {
  const float* a;
  const float* b;
  const float* bias;
  float* out;
  int m, n, k;
  int tiles_n;   // tiles along N (grid.x = tiles_n * tiles_m)
  int splits;    // cluster size along grid.y
  int kchunk;    // K elements per split (a multiple of kF32BK)
};

template <bool kBKMajor>
__global__ void __launch_bounds__(kF32Threads)
    gemm_f32_cluster_kernel(const F32GemmArgs p) {
  DLI_PDL_ENTRY();
  extern __shared__ __align__(16) float f32_smem[];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;  // 16 x 16 threads: 8 columns x 4 rows each
  const int tile_n = blockIdx.x % p.tiles_n, tile_m = blockIdx.x / p.tiles_n;
  const int m0 = tile_m * kF32BM, n0 = tile_n * kF32BN;
  const int split = blockIdx.y;
  const int k_begin = split * p.kchunk;
  const int k_end = min(p.k, k_begin + p.kchunk);

  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  // register staging of the next K slice (global -> registers -> shared)
  float4 ra, rb[2];
  auto fetch = [&](int k0) {
    {  // A: 64 rows x 16 k, one float4 per thread
      const int r = tid >> 2, kq = (tid & 3) * 4;
      const int gr = m0 + r, gk = k0 + kq;
      ra = (gr < p.m && gk < k_end) ? *reinterpret_cast<const float4*>(p.a + static_cast<int64_t>(gr) * p.k + gk)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int idx = tid + h * kF32Threads;
      if constexpr (kBKMajor) {  // B [N,K]: 128 rows x 16 k
        const int r = idx >> 2, kq = (idx & 3) * 4;
        const int gn = n0 + r, gk = k0 + kq;
        rb[h] = (gn < p.n && gk < k_end) ? *reinterpret_cast<const float4*>(p.b + static_cast<int64_t>(gn) * p.k + gk)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
      } else {  // B [K,N]: 16 k rows x 128 columns
        const int kr = idx >> 5, nq = (idx & 31) * 4;
        const int gk = k0 + kr, gn = n0 + nq;
        rb[h] = (gk < k_end && gn < p.n) ? *reinterpret_cast<const float4*>(p.b + static_cast<int64_t>(gk) * p.n + gn)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  auto stash = [&](int buf) {
    float* as = f32_smem + buf * kF32StageFloats;
    float* bs = as + kF32BK * kF32AStride;
    {
      const int r = tid >> 2, kq = (tid & 3) * 4;
      as[(kq + 0) * kF32AStride + r] = ra.x;
      as[(kq + 1) * kF32AStride + r] = ra.y;
      as[(kq + 2) * kF32AStride + r] = ra.z;
      as[(kq + 3) * kF32AStride + r] = ra.w;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int idx = tid + h * kF32Threads;
      if constexpr (kBKMajor) {
        const int r = idx >> 2, kq = (idx & 3) * 4;
        bs[(kq + 0) * kF32BStride + r] = rb[h].x;
        bs[(kq + 1) * kF32BStride + r] = rb[h].y;
        bs[(kq + 2) * kF32BStride + r] = rb[h].z;
        bs[(kq + 3) * kF32BStride + r] = rb[h].w;
      } else {
        const int kr = idx >> 5, nq = (idx & 31) * 4;
        *reinterpret_cast<float4*>(bs + kr * kF32BStride + nq) = rb[h];
      }
    }
  };

  const int slices = (k_end - k_begin + kF32BK - 1) / kF32BK;
  if (slices > 0) {
    fetch(k_begin);
    stash(0);
  }
  __syncthreads();
  for (int s = 0; s < slices; ++s) {
    const int buf = s & 1;
    if (s + 1 < slices) fetch(k_begin + (s + 1) * kF32BK);  // loads in flight during the FFMAs
    const float* as = f32_smem + buf * kF32StageFloats;
    const float* bs = as + kF32BK * kF32AStride;
#pragma unroll
    for (int kk = 0; kk < kF32BK; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(as + kk * kF32AStride + ty * 4);
      const float4 b0 = *reinterpret_cast<const float4*>(bs + kk * kF32BStride + tx * 8);
      const float4 b1 = *reinterpret_cast<const float4*>(bs + kk * kF32BStride + tx * 8 + 4);
      const float a4[4] = {av.x, av.y, av.z, av.w};
      const float b8[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a4[i], b8[j], acc[i][j]);
    }
    if (s + 1 < slices) stash(buf ^ 1);
    __syncthreads();
  }

  auto store = [&](int row, int col0, const float* v) {
    if (row >= p.m) return;
    float* dst = p.out + static_cast<int64_t>(row) * p.n + col0;
    if (col0 + 8 <= p.n && (p.n & 3) == 0) {
      float4 o0 = make_float4(v[0], v[1], v[2], v[3]), o1 = make_float4(v[4], v[5], v[6], v[7]);
      if (p.bias) {
        const float4 c0 = *reinterpret_cast<const float4*>(p.bias + col0);
        const float4 c1 = *reinterpret_cast<const float4*>(p.bias + col0 + 4);
        o0.x += c0.x; o0.y += c0.y; o0.z += c0.z; o0.w += c0.w;
        o1.x += c1.x; o1.y += c1.y; o1.z += c1.z; o1.w += c1.w;
      }
      *reinterpret_cast<float4*>(dst) = o0;
      *reinterpret_cast<float4*>(dst + 4) = o1;
    } else {
      for (int j = 0; j < 8 && col0 + j < p.n; ++j) dst[j] = v[j] + (p.bias ? p.bias[col0 + j] : 0.f);
    }
  };

  if (p.splits == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) store(m0 + ty * 4 + i, n0 + tx * 8, acc[i]);
    return;
  }
  // split-K: partial tile into this CTA's shared memory, then a cluster reduction
  float* red = f32_smem;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float* row = red + (ty * 4 + i) * kF32RedStride + tx * 8;
    *reinterpret_cast<float4*>(row) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    *reinterpret_cast<float4*>(row + 4) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
  }
  cluster_sync();
  const int S = p.splits;
  const int rows_per = (kF32BM + S - 1) / S;
  const uint32_t red_local = static_cast<uint32_t>(__cvta_generic_to_shared(red));
  // rank `split` sums rows [split*rows_per, ...) of every rank's partial, 8 columns per thread
  for (int q = tid; q < rows_per * (kF32BN / 8); q += kF32Threads) {
    const int rr = split * rows_per + q / (kF32BN / 8);
    const int c8 = (q % (kF32BN / 8)) * 8;
    if (rr >= kF32BM) continue;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < S; ++r) {
      const uint32_t off = static_cast<uint32_t>((rr * kF32RedStride + c8) * 4);
      const float4 x0 = ld_dsmem_f4(mapa_shared(red_local + off, r));
      const float4 x1 = ld_dsmem_f4(mapa_shared(red_local + off + 16, r));
      v[0] += x0.x; v[1] += x0.y; v[2] += x0.z; v[3] += x0.w;
      v[4] += x1.x; v[5] += x1.y; v[6] += x1.z; v[7] += x1.w;
    }
    store(m0 + rr, n0 + c8, v);
  }
  cluster_sync();  // every rank's shared memory stays alive until all reads are done
}

// ---- host helpers ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// K-major 2-D map over [rows, k] with row stride `ld` elements, box {64, box_rows}.
dli_status make_kmajor_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int64_t ld,
                           int box_rows, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(DLI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DLI_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
  return DLI_OK;
}

// MN-major 2-D map over [k, cols] (cols contiguous, row stride `ld` elements),
// box {64 columns, kBK rows}: the right operand of matmul.
dli_status make_mnmajor_map(CUtensorMap* map, const void* base, int64_t k, int64_t cols, int64_t ld, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(DLI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(k)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(kBK)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DLI_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
  return DLI_OK;
}

// Pipeline depth per tile width. Narrow (decode, swap-AB) tiles use ~100 KB of
// shared memory so two CTAs share an SM: one CTA's prologue and split-K
// epilogue overlap the other's weight streaming. Wide tiles fill ~200 KB.
// DLI_SM100_GEMM_DEEP=1 gives narrow tiles one ~200 KB CTA per SM instead.
bool gemm_deep() {
  static const bool deep = tuning_knob("GEMM_DEEP", 0) != 0;
  return deep;
}
int stages_for(int bn) {
  if (bn >= 256) return 4;
  if (bn >= 128) return 6;
  if (bn >= 64) return gemm_deep() ? 7 : 3;
  return gemm_deep() ? 10 : 4;
}

template <typename T, int BN, int STAGES>
dli_status launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const TcParams& p, int splits,
                     cudaStream_t stream) {
  using L = TcLayout<BN, STAGES>;
  auto kernel = tcgen05_gemm_kernel<T, BN, STAGES>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kernel), L::kBytes, "tcgen05 gemm");
  if (st != DLI_OK) return st;
  dim3 grid(static_cast<unsigned>(p.tiles_i * p.tiles_j), static_cast<unsigned>(splits));
  launch_pdl_cluster(kernel, grid, dim3(kGemmThreads), L::kBytes, stream,
                     static_cast<unsigned>(splits), ma, mb, p);
  return check_launch("tcgen05 gemm");
}

template <typename T>
dli_status launch_tc_persistent(const CUtensorMap& ma, const CUtensorMap& mb, const TcParams& p,
                                cudaStream_t stream) {
  using L = PersistentLayout<4>;
  auto kernel = tcgen05_gemm_persistent_kernel<T, 4>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kernel), L::kBytes, "tcgen05 gemm");
  if (st != DLI_OK) return st;
  const int tiles = p.tiles_i * p.tiles_j;
  dim3 grid(static_cast<unsigned>(std::min(tiles, sm_count())));
  launch_pdl(kernel, grid, dim3(kGemmThreads), L::kBytes, stream, ma, mb, p);
  return check_launch("tcgen05 gemm");
}

template <typename T, int BN, int STAGES>
dli_status launch_tc_streamk(const CUtensorMap& ma, const CUtensorMap& mb, const TcParams& p, int ctas,
                             cudaStream_t stream) {
  using L = StreamKLayout<BN, STAGES>;
  auto kernel = tcgen05_gemm_streamk_kernel<T, BN, STAGES>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kernel), L::kBytes, "tcgen05 gemm");
  if (st != DLI_OK) return st;
  launch_pdl(kernel, dim3(static_cast<unsigned>(ctas)), dim3(kGemmThreads), L::kBytes, stream, ma, mb, p);
  return check_launch("tcgen05 gemm (stream-K)");
}

// Stream-K stage counts: two CTAs per SM (~110 KB each) at tile widths 32 and 64.
constexpr int kStreamKStages32 = 5;
constexpr int kStreamKStages64 = 3;

// Persistent double-buffered kernel for many-tile, un-split, row-per-thread
// epilogues (prefill projections, conv); DLI_SM100_GEMM_PERSISTENT=0 disables it.
bool use_persistent(const GemmPlan& plan, int epilogue) {
  static const bool on = tuning_knob("GEMM_PERSISTENT", 1) != 0;
  return on && plan.bn == 256 && plan.splits == 1 && epilogue != kEpiTransposed && epilogue != kEpiGluT &&
         static_cast<int64_t>(plan.tiles_i) * plan.tiles_j > sm_count();
}

template <typename T>
dli_status launch_tc_bn(int bn, int stages, const CUtensorMap& ma, const CUtensorMap& mb,
                        const TcParams& p, int splits, cudaStream_t stream) {
  switch (bn) {
    case 32: return stages == 10 ? launch_tc<T, 32, 10>(ma, mb, p, splits, stream)
                                 : launch_tc<T, 32, 4>(ma, mb, p, splits, stream);
    case 64: return stages == 7 ? launch_tc<T, 64, 7>(ma, mb, p, splits, stream)
                                : launch_tc<T, 64, 3>(ma, mb, p, splits, stream);
    case 128: return launch_tc<T, 128, 6>(ma, mb, p, splits, stream);
    case 256: return launch_tc<T, 256, 4>(ma, mb, p, splits, stream);
  }
  return fail(DLI_ERR_UNSUPPORTED, "gemm: unsupported tile width");
}

// Occupancy of one kernel configuration: CTAs per SM (cluster == 1) or
// resident clusters of `cluster` CTAs (clusters are placed within a GPC, so
// the latter is below sm_count * CTAs-per-SM / cluster for clusters above 2).
// The calculator reports one CTA per SM for any kernel that allocates tensor
// memory, while the hardware co-schedules as many as shared memory, registers
// and the 512 TMEM columns allow (two 101 KB GEMM CTAs of 32-256 columns run
// side by side on B200). The query therefore runs on a proxy kernel with this
// configuration's block size and shared memory and no TMEM use; registers
// (<= 96 per thread here) never bind before shared memory does.
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_occupancy_proxy(int* sink) {
  extern __shared__ int proxy_smem[];
  if (sink != nullptr) sink[threadIdx.x] = proxy_smem[threadIdx.x];
}

int query_occupancy(int smem_bytes, int cluster) {
  // the proxy serves every configuration: set its limit to this one's size
  if (cudaFuncSetAttribute(gemm_occupancy_proxy, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (cluster <= 1) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemm_occupancy_proxy, kGemmThreads, smem_bytes) !=
        cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return n;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, static_cast<unsigned>(cluster), 1);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = static_cast<unsigned>(cluster);
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_occupancy_proxy, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Rings of the fp32 split kernel at tile width 32: two raw and two converted
// stages (default), so the converter warps split K block k+1 while the MMAs of
// block k still read theirs; DLI_SM100_GEMM_F32X3_CS=1 keeps three raw stages
// and one converted stage, where each block's conversion waited for the
// previous block's MMAs. Wider tiles fit only one converted stage.
bool f32x3_two_cv_stages() {
  static const bool two = tuning_knob("GEMM_F32X3_CS", 2) != 1;
  return two;
}

int layout_bytes(int bn, int stages) {
  switch (bn * 100 + stages) {
    case 3204: return TcLayout<32, 4>::kBytes;
    case 3210: return TcLayout<32, 10>::kBytes;
    case 6403: return TcLayout<64, 3>::kBytes;
    case 6407: return TcLayout<64, 7>::kBytes;
    case 12806: return TcLayout<128, 6>::kBytes;
    case 25604: return TcLayout<256, 4>::kBytes;
    // stages 0: the fp32 split-bf16 kernel's rings at that tile width
    case 3200: return f32x3_two_cv_stages() ? F32x3Layout<32, 2, 2>::kBytes : F32x3Layout<32, 3, 1>::kBytes;
    case 6400: return F32x3Layout<64, 3, 1>::kBytes;
    case 12800: return F32x3Layout<128, 2, 1>::kBytes;
    default: return 0;
  }
}

}  // namespace

int gemm_occupancy(int bn, int stages, int cluster) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const auto key = std::make_tuple(dev, bn, stages, cluster);
  std::lock_guard<std::mutex> lock(mu);  // also serialises the proxy's attribute changes
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  const int bytes = layout_bytes(bn, stages);
  const int n = bytes > 0 ? query_occupancy(bytes, cluster) : 0;
  cache[key] = n;
  return n;
}

GemmPlan plan_tn_gemm(int64_t rows_a, int64_t rows_b, int64_t k, dli_dtype dtype, bool allow_split) {
  GemmPlan plan;
  const bool tc_type = dtype == DLI_DTYPE_BF16 || dtype == DLI_DTYPE_F16;
  if (!tc_type || k % 8 != 0 || k <= 0 || rows_a <= 0 || rows_b <= 0 || rows_a > (1ll << 31) ||
      rows_b > (1ll << 31))
    return plan;
  plan.tcgen05 = true;
  if (rows_b <= 32) plan.bn = 32;
  else if (rows_b <= 64) plan.bn = 64;
  else if (rows_b <= 128) plan.bn = 128;
  else plan.bn = (rows_b % 256 == 0 || rows_b >= 2048) ? 256 : 128;
  plan.stages = stages_for(plan.bn);
  plan.tiles_i = static_cast<int>(ceil_div(rows_a, kBM));
  plan.tiles_j = static_cast<int>(ceil_div(rows_b, plan.bn));
  plan.kblocks = static_cast<int>(ceil_div(k, kBK));
  plan.splits = 1;
  const int64_t tiles = static_cast<int64_t>(plan.tiles_i) * plan.tiles_j;
  const int slots = sm_count() * std::max(1, gemm_occupancy(plan.bn, plan.stages, 1));
  // When the tiles alone cannot fill the SMs, split K over a thread-block cluster
  // of S <= 8 CTAs per tile (reduced through distributed shared memory, so splits
  // cost no global traffic): the largest S whose clusters all fit on the GPU at
  // once, each split keeping >= 3 K blocks.
  static const int kForceSplits = tuning_knob("GEMM_SPLITS", 0);  // fixed S (launch-shape sweeps)
  if (allow_split && tiles < slots && kForceSplits > 0) {
    plan.splits = std::max(1, std::min({kForceSplits, 8, plan.kblocks / 2}));
  } else if (allow_split && tiles < slots) {
    for (int s = 8; s >= 2; --s) {
      if (plan.kblocks < 3 * s || tiles * s > slots) continue;
      if (tiles <= gemm_occupancy(plan.bn, plan.stages, s)) {
        plan.splits = s;
        break;
      }
    }
  }
  plan.workspace = 0;
  return plan;
}

GemmPlan plan_streamk(GemmPlan plan) {
  static const bool on = tuning_knob("GEMM_STREAMK", 0) != 0;  // off: measured slower than cluster split-K
  if (!on || !plan.tcgen05 || (plan.bn != 32 && plan.bn != 64) || plan.kblocks < 2) return plan;
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> occ_cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return plan;
  }
  int occ = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(dev, plan.bn);
    auto it = occ_cache.find(key);
    if (it != occ_cache.end()) {
      occ = it->second;
    } else {
      const int bytes = plan.bn == 32 ? StreamKLayout<32, kStreamKStages32>::kBytes
                                      : StreamKLayout<64, kStreamKStages64>::kBytes;
      occ = query_occupancy(bytes, 1);
      occ_cache[key] = occ;
    }
  }
  if (occ <= 0) return plan;
  const int64_t slots = static_cast<int64_t>(sm_count()) * std::min(occ, 2);
  const int64_t tiles = static_cast<int64_t>(plan.tiles_i) * plan.tiles_j;
  if (tiles % slots == 0) return plan;  // whole waves already: the data-parallel launch is balanced
  const int64_t units = tiles * plan.kblocks;
  const int64_t ctas = std::min<int64_t>(slots, units);
  plan.streamk_ctas = static_cast<int>(ctas);
  plan.splits = 1;
  const size_t partial = static_cast<size_t>(ctas) * 2 * kBM * plan.bn * sizeof(float);
  plan.workspace = (partial + static_cast<size_t>(tiles) * sizeof(int) + 255) / 256 * 256;
  return plan;
}

dli_status run_tn_gemm_tcgen05(const void* a, const void* b, const void* bias, void* out,
                               int64_t rows_a, int64_t rows_b, int64_t k, int64_t lda,
                               int64_t ldb, int64_t ldo, int epilogue, int64_t ohw,
                               dli_dtype dtype, const GemmPlan& plan, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream, bool const_a,
                               bool const_b, int64_t glu_cols, bool out_f32, bool b_mn) {
  if (!plan.tcgen05) return fail(DLI_ERR_UNSUPPORTED, "gemm: shape not served by tcgen05");
  if (b_mn && (plan.bn < 64 || plan.streamk_ctas > 0 || epilogue != kEpiRowMajor))
    return fail(DLI_ERR_UNSUPPORTED, "gemm: MN-major B needs a row-major plan with tile width >= 64");
  if (out_f32 && epilogue != kEpiRowMajor && epilogue != kEpiTransposed)
    return fail(DLI_ERR_UNSUPPORTED, "gemm: float32 output only for plain row-major/transposed epilogues");
  if (!aligned(a, 16) || !aligned(b, 16) || lda % 8 != 0 || ldb % 8 != 0)
    return fail(DLI_ERR_UNSUPPORTED, "gemm: TMA needs 16-byte aligned operands and row strides");
  if (plan.streamk_ctas > 0 && (workspace == nullptr || workspace_bytes < plan.workspace ||
                                epilogue == kEpiRowMajor || epilogue == kEpiNchw || epilogue == kEpiGlu))
    return fail(DLI_ERR_WORKSPACE, "gemm: the stream-K plan needs a zero-filled workspace of " +
                                       std::to_string(plan.workspace) + " bytes");
  const bool bf16 = dtype == DLI_DTYPE_BF16;
  CUtensorMap ma, mb;
  dli_status st = make_kmajor_map(&ma, a, rows_a, k, lda, kBM, bf16);
  if (st != DLI_OK) return st;
  st = b_mn ? make_mnmajor_map(&mb, b, k, rows_b, ldb, bf16) : make_kmajor_map(&mb, b, rows_b, k, ldb, plan.bn, bf16);
  if (st != DLI_OK) return st;
  TcParams p{};
  p.rows_a = static_cast<int>(rows_a);
  p.rows_b = static_cast<int>(rows_b);
  p.tiles_i = plan.tiles_i;
  p.tiles_j = plan.tiles_j;
  p.kblocks = plan.kblocks;
  p.splits = plan.splits;
  p.epilogue = epilogue;
  p.ldo = ldo;
  p.ohw = ohw > 0 ? ohw : 1;
  p.out_vec = aligned(out, 16) ? 1 : 0;
  p.bias = bias;
  p.out = out;
  p.err = device_error_word();
  p.const_a = const_a ? 1 : 0;
  p.const_b = const_b ? 1 : 0;
  p.glu_cols = static_cast<int>(glu_cols);
  p.out_f32 = out_f32 ? 1 : 0;
  p.b_mn = b_mn ? 1 : 0;
  if (plan.streamk_ctas > 0) {
    p.sk_part = static_cast<float*>(workspace);
    p.sk_count = reinterpret_cast<int*>(static_cast<char*>(workspace) +
                                        static_cast<size_t>(plan.streamk_ctas) * 2 * kBM * plan.bn * sizeof(float));
    if (plan.bn == 32)
      return bf16 ? launch_tc_streamk<__nv_bfloat16, 32, kStreamKStages32>(ma, mb, p, plan.streamk_ctas, stream)
                  : launch_tc_streamk<__half, 32, kStreamKStages32>(ma, mb, p, plan.streamk_ctas, stream);
    return bf16 ? launch_tc_streamk<__nv_bfloat16, 64, kStreamKStages64>(ma, mb, p, plan.streamk_ctas, stream)
                : launch_tc_streamk<__half, 64, kStreamKStages64>(ma, mb, p, plan.streamk_ctas, stream);
  }
  if (use_persistent(plan, epilogue))
    return bf16 ? launch_tc_persistent<__nv_bfloat16>(ma, mb, p, stream) : launch_tc_persistent<__half>(ma, mb, p, stream);
  if (bf16) return launch_tc_bn<__nv_bfloat16>(plan.bn, plan.stages, ma, mb, p, plan.splits, stream);
  return launch_tc_bn<__half>(plan.bn, plan.stages, ma, mb, p, plan.splits, stream);
}

template <typename T, int BN, int STAGES>
dli_status launch_conv(const CUtensorMap& mb, const TcParams& p, const void* x, const ConvGeom& g, int splits,
                       cudaStream_t stream) {
  using L = TcLayout<BN, STAGES>;
  constexpr int kBytes = L::kBytes + STAGES * 8 + 2 * kBK * 8 + 64;  // + patch barriers, k tables, votes
  auto kernel = tcgen05_conv_kernel<T, BN, STAGES>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kernel), kBytes, "tcgen05 conv");
  if (st != DLI_OK) return st;
  dim3 grid(static_cast<unsigned>(p.tiles_i * p.tiles_j), static_cast<unsigned>(splits));
  launch_pdl_cluster(kernel, grid, dim3(kConvThreads), kBytes, stream, static_cast<unsigned>(splits), mb, p,
                     static_cast<const T*>(x), g);
  return check_launch("tcgen05 conv");
}

template <typename T>
dli_status launch_conv_bn(int bn, int stages, const CUtensorMap& mb, const TcParams& p, const void* x,
                          const ConvGeom& g, int splits, cudaStream_t stream) {
  switch (bn) {
    case 32: return stages == 10 ? launch_conv<T, 32, 10>(mb, p, x, g, splits, stream)
                                 : launch_conv<T, 32, 4>(mb, p, x, g, splits, stream);
    case 64: return stages == 7 ? launch_conv<T, 64, 7>(mb, p, x, g, splits, stream)
                                : launch_conv<T, 64, 3>(mb, p, x, g, splits, stream);
    case 128: return launch_conv<T, 128, 6>(mb, p, x, g, splits, stream);
    case 256: return launch_conv<T, 256, 4>(mb, p, x, g, splits, stream);
  }
  return fail(DLI_ERR_UNSUPPORTED, "conv: unsupported tile width");
}

// fp32 2-D map over [outer, inner] (row stride `ld` floats), 128B-swizzled
// boxes of 32 x box_outer: K-major operands (inner = K) and MN-major B (inner = N).
dli_status make_f32_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t ld,
                        int box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(DLI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  const cuuint32_t box[2] = {32u, static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DLI_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
  return DLI_OK;
}

template <int BN, int RS, int CS>
dli_status launch_f32x3(const CUtensorMap& ma, const CUtensorMap& mb, const TcParams& p, int splits,
                        cudaStream_t stream) {
  using L = F32x3Layout<BN, RS, CS>;
  auto kernel = tcgen05_gemm_f32x3_kernel<BN, RS, CS>;
  const dli_status st = ensure_smem(reinterpret_cast<const void*>(kernel), L::kBytes, "fp32 tcgen05 gemm");
  if (st != DLI_OK) return st;
  dim3 grid(static_cast<unsigned>(p.tiles_i * p.tiles_j), static_cast<unsigned>(splits));
  launch_pdl_cluster(kernel, grid, dim3(kF32SplitThreads), L::kBytes, stream, static_cast<unsigned>(splits), ma, mb,
                     p);
  return check_launch("fp32 tcgen05 gemm");
}

dli_status run_conv_implicit_tcgen05(const void* x, const void* w_kmajor, int64_t kp, const void* bias, void* out,
                                     const ConvGeom& g, dli_dtype dtype, cudaStream_t stream, bool const_w) {
  const bool bf16 = dtype == DLI_DTYPE_BF16;
  if (!bf16 && dtype != DLI_DTYPE_F16) return fail(DLI_ERR_UNSUPPORTED, "conv: bfloat16/float16 only");
  const int64_t m = static_cast<int64_t>(g.n) * g.oh * g.ow;
  const GemmPlan plan = plan_tn_gemm(m, g.oc, kp, dtype, true);
  if (!plan.tcgen05 || kp % 8 != 0 || !aligned(w_kmajor, 16))
    return fail(DLI_ERR_UNSUPPORTED, "conv: shape not served by the implicit tcgen05 path");
  CUtensorMap mb;
  dli_status st = make_kmajor_map(&mb, w_kmajor, g.oc, kp, kp, plan.bn, bf16);
  if (st != DLI_OK) return st;
  TcParams p{};
  p.rows_a = static_cast<int>(m);
  p.rows_b = g.oc;
  p.tiles_i = plan.tiles_i;
  p.tiles_j = plan.tiles_j;
  p.kblocks = plan.kblocks;
  p.splits = plan.splits;
  p.epilogue = kEpiNchw;
  p.ldo = 0;
  p.ohw = static_cast<int64_t>(g.oh) * g.ow;
  p.out_vec = 0;
  p.bias = bias;
  p.out = out;
  p.err = device_error_word();
  p.const_b = const_w ? 1 : 0;
  return bf16 ? launch_conv_bn<__nv_bfloat16>(plan.bn, plan.stages, mb, p, x, g, plan.splits, stream)
              : launch_conv_bn<__half>(plan.bn, plan.stages, mb, p, x, g, plan.splits, stream);
}

// fp32 D = A * B^T (+ bias) on tcgen05 through the three-term bf16 split: A [rows_a,
// K] K-major; B [rows_b, K] K-major, or [K, rows_b] MN-major (b_mn). True when
// it served the call (16-byte aligned operands, K and the leading dimensions
// multiples of 4 floats, DLI_SM100_GEMM_F32X3 not 0); *status then holds the
// launch result.
bool try_gemm_f32x3(const void* a, const void* b, const void* bias, void* out, int64_t rows_a, int64_t rows_b,
                    int64_t k, int64_t ldb, int64_t ldo, int epilogue, bool b_mn, cudaStream_t stream,
                    dli_status* status) {
  static const bool on = tuning_knob("GEMM_F32X3", 1) != 0;
  if (!on || k % 4 != 0 || ldb % 4 != 0 || !aligned(a, 16) || !aligned(b, 16) || rows_a <= 0 || rows_b <= 0 ||
      rows_a > (1ll << 30) || rows_b > (1ll << 30) || k > (1ll << 30))
    return false;
  const int bn = (rows_b <= 32 && !b_mn) ? 32 : rows_b <= 64 ? 64 : 128;
  const int stages_code = 0;
  GemmPlan plan;
  plan.bn = bn;
  plan.tiles_i = static_cast<int>(ceil_div(rows_a, kBM));
  plan.tiles_j = static_cast<int>(ceil_div(rows_b, bn));
  plan.kblocks = static_cast<int>(ceil_div(k, kBK));
  if (static_cast<int64_t>(plan.tiles_i) * plan.tiles_j > 0x7fffffff) return false;
  const int64_t tiles = static_cast<int64_t>(plan.tiles_i) * plan.tiles_j;
  const int slots = sm_count() * std::max(1, gemm_occupancy(bn, stages_code, 1));
  plan.splits = 1;
  if (tiles < slots) {  // the bf16 plan's rule: largest cluster split that fits, >= 3 K blocks each
    for (int s = 8; s >= 2; --s) {
      if (plan.kblocks < 3 * s || tiles * s > slots) continue;
      if (tiles <= gemm_occupancy(bn, stages_code, s)) {
        plan.splits = s;
        break;
      }
    }
  }
  CUtensorMap ma, mb;
  *status = make_f32_map(&ma, a, k, rows_a, k, kBM);
  if (*status == DLI_OK)
    *status = b_mn ? make_f32_map(&mb, b, rows_b, k, ldb, kBK) : make_f32_map(&mb, b, k, rows_b, ldb, bn);
  if (*status != DLI_OK) return true;
  TcParams p{};
  p.rows_a = static_cast<int>(rows_a);
  p.rows_b = static_cast<int>(rows_b);
  p.tiles_i = plan.tiles_i;
  p.tiles_j = plan.tiles_j;
  p.kblocks = plan.kblocks;
  p.splits = plan.splits;
  p.epilogue = epilogue;
  p.ldo = ldo;
  p.ohw = 1;
  p.out_vec = 0;
  p.bias = bias;
  p.out = out;
  p.err = device_error_word();
  p.out_f32 = 1;
  p.bias_f32 = 1;
  p.b_mn = b_mn ? 1 : 0;
  switch (bn) {
    case 32:
      *status = f32x3_two_cv_stages() ? launch_f32x3<32, 2, 2>(ma, mb, p, plan.splits, stream)
                                      : launch_f32x3<32, 3, 1>(ma, mb, p, plan.splits, stream);
      break;
    case 64: *status = launch_f32x3<64, 3, 1>(ma, mb, p, plan.splits, stream); break;
    default: *status = launch_f32x3<128, 2, 1>(ma, mb, p, plan.splits, stream); break;
  }
  return true;
}

// Cluster split-K fp32 GEMM: true when it served the call (fp32, 16-byte aligned
// operands, K and the [K,N] row stride multiples of 4 elements).
bool try_gemm_f32(const void* a, const void* b, const void* bias, void* out, int64_t m, int64_t n, int64_t k,
                  bool b_kmajor, cudaStream_t stream, dli_status* status) {
  static const bool on = tuning_knob("GEMM_F32", 1) != 0;
  if (!on || k % 4 != 0 || (!b_kmajor && n % 4 != 0) || !aligned(a, 16) || !aligned(b, 16) || !aligned(out, 16) ||
      (bias && !aligned(bias, 16)) || m > (1 << 30) || n > (1 << 30) || k > (1 << 30))
    return false;
  const int64_t tiles = ceil_div(n, kF32BN) * ceil_div(m, kF32BM);
  if (tiles > 0x7fffffff) return false;
  // splits: enough CTAs for two per SM, each split keeping >= 256 K elements
  const int64_t target = 2 * static_cast<int64_t>(sm_count());
  int splits = static_cast<int>(std::min<int64_t>(8, std::max<int64_t>(1, ceil_div(target, tiles))));
  splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(splits, k / 256)));
  const int kchunk = static_cast<int>(ceil_div(ceil_div(k, splits), kF32BK) * kF32BK);
  splits = static_cast<int>(ceil_div(k, kchunk));
  F32GemmArgs args{static_cast<const float*>(a), static_cast<const float*>(b), static_cast<const float*>(bias),
                   static_cast<float*>(out), static_cast<int>(m), static_cast<int>(n), static_cast<int>(k),
                   static_cast<int>(ceil_div(n, kF32BN)), splits, kchunk};
  auto kern = b_kmajor ? gemm_f32_cluster_kernel<true> : gemm_f32_cluster_kernel<false>;
  *status = ensure_smem(reinterpret_cast<const void*>(kern), kF32SmemBytes, "fp32 gemm");
  if (*status != DLI_OK) return true;
  launch_pdl_cluster(kern, dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(splits)), dim3(kF32Threads),
                     kF32SmemBytes, stream, static_cast<unsigned>(splits), args);
  *status = check_launch("fp32 gemm");
  return true;
}

dli_status run_gemm_simt(const void* a, const void* b, const void* bias, void* out, int64_t m,
                         int64_t n, int64_t k, bool b_kmajor, dli_dtype dtype,
                         cudaStream_t stream) {
  if (dtype == DLI_DTYPE_F32) {
    dli_status st = DLI_OK;
    if (try_gemm_f32(a, b, bias, out, m, n, k, b_kmajor, stream, &st)) return st;
  }
  if (ceil_div(m, kSimtTile) > 65535) return fail(DLI_ERR_UNSUPPORTED, "gemm: too many rows for SIMT path");
  dim3 grid(static_cast<unsigned>(ceil_div(n, kSimtTile)), static_cast<unsigned>(ceil_div(m, kSimtTile)));
  dli_status st = dispatch_float(dtype, "gemm", [&](auto tag) {
    using T = decltype(tag);
    if (b_kmajor)
      launch_pdl(gemm_simt_kernel<T, true>, grid, dim3(256), 0, stream, (const T*)a, (const T*)b,
                 (const T*)bias, (T*)out, m, n, k);
    else
      launch_pdl(gemm_simt_kernel<T, false>, grid, dim3(256), 0, stream, (const T*)a, (const T*)b,
                 (const T*)bias, (T*)out, m, n, k);
  });
  if (st != DLI_OK) return st;
  return check_launch("simt gemm");
}

}  // namespace dli_sm100

using namespace dli_sm100;

namespace {
// Activation rows at or below this count run swap-AB (weights on the MMA M side).
constexpr int64_t kSwapRows = 128;

// The tcgen05 plan of a linear: swap-AB decode problems take the stream-K plan
// when the caller's workspace holds it (and the cluster split-K plan otherwise).
GemmPlan linear_plan(int64_t m, int64_t n, int64_t k, dli_dtype dtype, size_t workspace_bytes, bool query) {
  if (m > kSwapRows) return plan_tn_gemm(m, n, k, dtype, true);
  const GemmPlan base = plan_tn_gemm(n, m, k, dtype, true);
  const GemmPlan sk = plan_streamk(base);
  return (sk.streamk_ctas > 0 && (query || workspace_bytes >= sk.workspace)) ? sk : base;
}
}  // namespace

extern "C" size_t dli_sm100_linear_workspace_size(int64_t m, int64_t n, int64_t k, dli_dtype dtype) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const GemmPlan plan = linear_plan(m, n, k, dtype, 0, true);
  return plan.tcgen05 ? plan.workspace : 0;
}

extern "C" dli_status dli_sm100_linear(const void* x, const void* w, const void* bias, void* y,
                                       int64_t m, int64_t n, int64_t k, dli_dtype dtype,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 0 || n <= 0 || k <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "linear: bad sizes");
  if (!is_float_dtype(dtype)) return fail(DLI_ERR_INVALID_ARGUMENT, "linear expects a float dtype");
  if (m == 0) return ok();
  if (!x || !w || !y) return fail(DLI_ERR_INVALID_ARGUMENT, "linear: null pointer");
  const bool swap = m <= kSwapRows;
  if (dtype == DLI_DTYPE_F32) {
    dli_status st = DLI_OK;
    const bool served = swap ? try_gemm_f32x3(w, x, bias, y, n, m, k, k, n, kEpiTransposed, false, as_stream(stream), &st)
                             : try_gemm_f32x3(x, w, bias, y, m, n, k, k, n, kEpiRowMajor, false, as_stream(stream), &st);
    if (served) return st;
  }
  const GemmPlan plan = linear_plan(m, n, k, dtype, workspace ? workspace_bytes : 0, false);
  const bool tma_ok = aligned(x, 16) && aligned(w, 16);
  if (plan.tcgen05 && tma_ok) {
    if (swap)
      return run_tn_gemm_tcgen05(w, x, bias, y, n, m, k, k, k, n, kEpiTransposed, 0, dtype, plan,
                                 workspace, workspace_bytes, as_stream(stream), true, false);
    return run_tn_gemm_tcgen05(x, w, bias, y, m, n, k, k, k, n, kEpiRowMajor, 0, dtype, plan,
                               workspace, workspace_bytes, as_stream(stream), false, true);
  }
  return run_gemm_simt(x, w, bias, y, m, n, k, true, dtype, as_stream(stream));
}

extern "C" dli_status dli_sm100_linear_ex(const void* x, const void* w, const void* bias, void* y, int64_t m,
                                          int64_t n, int64_t k, dli_dtype dtype, dli_dtype out_dtype,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  if (out_dtype == dtype)
    return dli_sm100_linear(x, w, bias, y, m, n, k, dtype, workspace, workspace_bytes, stream);
  if (m < 0 || n <= 0 || k <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "linear_ex: bad sizes");
  if ((dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16) || out_dtype != DLI_DTYPE_F32)
    return fail(DLI_ERR_UNSUPPORTED, "linear_ex: only bfloat16/float16 operands with a float32 output");
  if (m == 0) return ok();
  if (!x || !w || !y) return fail(DLI_ERR_INVALID_ARGUMENT, "linear_ex: null pointer");
  if (!aligned(x, 16) || !aligned(w, 16) || k % 8 != 0)
    return fail(DLI_ERR_UNSUPPORTED, "linear_ex: 16-byte aligned operands and K % 8 == 0 expected");
  const bool swap = m <= kSwapRows;
  const GemmPlan plan = linear_plan(m, n, k, dtype, workspace ? workspace_bytes : 0, false);
  if (!plan.tcgen05) return fail(DLI_ERR_UNSUPPORTED, "linear_ex: shape not served by tcgen05");
  if (swap)
    return run_tn_gemm_tcgen05(w, x, bias, y, n, m, k, k, k, n, kEpiTransposed, 0, dtype, plan, workspace,
                               workspace_bytes, as_stream(stream), true, false, 0, true);
  return run_tn_gemm_tcgen05(x, w, bias, y, m, n, k, k, k, n, kEpiRowMajor, 0, dtype, plan, workspace,
                             workspace_bytes, as_stream(stream), false, true, 0, true);
}

extern "C" dli_status dli_sm100_linear_exchange_push(const void* x, const void* w, const void* bias, int64_t m,
                                                     int64_t n, int64_t k, dli_dtype dtype, void* const* buffers,
                                                     int tp, int rank, int64_t max_rows, int64_t row_elems,
                                                     void* stream) {
  const std::string name = "linear_exchange_push";
  if (m < 0 || n <= 0 || k <= 0 || max_rows <= 0 || row_elems <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, name + ": bad sizes");
  if (buffers == nullptr || tp < 1 || tp > kExchangeMaxRanks || rank < 0 || rank >= tp)
    return fail(DLI_ERR_INVALID_ARGUMENT, name + ": bad rank arguments");
  if (dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16)
    return fail(DLI_ERR_UNSUPPORTED, name + ": bfloat16/float16 only");
  if (m == 0) return ok();
  if (!x || !w) return fail(DLI_ERR_INVALID_ARGUMENT, name + ": null pointer");
  // Shape checks only (the same answer on every rank, so a caller that falls
  // back to the two-kernel path on DLI_ERR_UNSUPPORTED keeps the group in step):
  // a swap-AB decode tile whose K is split over a cluster (push reduction).
  if (m > kSwapRows || m > max_rows || n > row_elems || n % 8 != 0 || row_elems % 8 != 0 || k % 8 != 0)
    return fail(DLI_ERR_UNSUPPORTED, name + ": shape outside the fused exchange path");
  const GemmPlan plan = plan_tn_gemm(n, m, k, dtype, true);
  if (!plan.tcgen05 || plan.bn > 64 || plan.splits < 2)
    return fail(DLI_ERR_UNSUPPORTED, name + ": plan without a split-K push reduction");
  if (!aligned(x, 16) || !aligned(w, 16) || (bias && !aligned(bias, 2)))
    return fail(DLI_ERR_INVALID_ARGUMENT, name + ": 16-byte aligned operands expected");
  TcParams p{};
  for (int i = 0; i < tp; ++i) {
    if (buffers[i] == nullptr || !aligned(buffers[i], 256))
      return fail(DLI_ERR_INVALID_ARGUMENT, name + ": exchange buffers must be 256-byte aligned");
    p.xbuf[i] = static_cast<char*>(buffers[i]);
  }
  const bool bf16 = dtype == DLI_DTYPE_BF16;
  CUtensorMap ma, mb;
  dli_status st = make_kmajor_map(&ma, w, n, k, k, kBM, bf16);
  if (st != DLI_OK) return st;
  st = make_kmajor_map(&mb, x, m, k, k, plan.bn, bf16);
  if (st != DLI_OK) return st;
  p.rows_a = static_cast<int>(n);
  p.rows_b = static_cast<int>(m);
  p.tiles_i = plan.tiles_i;
  p.tiles_j = plan.tiles_j;
  p.kblocks = plan.kblocks;
  p.splits = plan.splits;
  p.epilogue = kEpiExchange;
  p.ohw = 1;
  p.bias = bias;
  p.out = nullptr;
  p.err = device_error_word();
  p.const_a = 1;
  p.xtp = tp;
  p.xrank = rank;
  p.xmax_rows = max_rows;
  p.xrow_words = row_elems * 2 / 4;
  return bf16 ? launch_tc_bn<__nv_bfloat16>(plan.bn, plan.stages, ma, mb, p, plan.splits, as_stream(stream))
              : launch_tc_bn<__half>(plan.bn, plan.stages, ma, mb, p, plan.splits, as_stream(stream));
}

extern "C" dli_status dli_sm100_linear_qkv_rotary_cache(
    const void* x, const void* wqkv, const void* bqkv, const float* cos_table, const float* sin_table,
    const int64_t* positions, void* q_out, void* cache_k, void* cache_v, int64_t batch, int64_t seq, int64_t k,
    int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t pairs, int64_t table_rows, int64_t capacity,
    dli_dtype dtype, void* stream) {
  const std::string name = "linear_qkv_rotary_cache";
  if (batch < 0 || seq < 0 || k <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0 ||
      pairs < 0 || pairs > head_dim / 2 || table_rows <= 0 || capacity <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, name + ": bad sizes");
  if (dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16)
    return fail(DLI_ERR_UNSUPPORTED, name + ": bfloat16/float16 only");
  const int64_t m = batch * seq, n = (q_heads + 2 * kv_heads) * head_dim;
  if (m == 0) return ok();
  if (!x || !wqkv || !cos_table || !sin_table || !positions || !q_out || !cache_k || !cache_v)
    return fail(DLI_ERR_INVALID_ARGUMENT, name + ": null pointer");
  // decode-sized calls whose K is split over a cluster (push reduction); others
  // take linear + dli_sm100_qkv_rotary_cache
  if (m > kSwapRows || k % 8 != 0 || n > (1 << 30))
    return fail(DLI_ERR_UNSUPPORTED, name + ": shape outside the fused path");
  const GemmPlan plan = plan_tn_gemm(n, m, k, dtype, true);
  if (!plan.tcgen05 || plan.bn > 64 || plan.splits < 2)
    return fail(DLI_ERR_UNSUPPORTED, name + ": plan without a split-K push reduction");
  if (!aligned(x, 16) || !aligned(wqkv, 16))
    return fail(DLI_ERR_UNSUPPORTED, name + ": 16-byte aligned operands expected");
  const bool bf16 = dtype == DLI_DTYPE_BF16;
  CUtensorMap ma, mb;
  dli_status st = make_kmajor_map(&ma, wqkv, n, k, k, kBM, bf16);
  if (st != DLI_OK) return st;
  st = make_kmajor_map(&mb, x, m, k, k, plan.bn, bf16);
  if (st != DLI_OK) return st;
  TcParams p{};
  p.rows_a = static_cast<int>(n);
  p.rows_b = static_cast<int>(m);
  p.tiles_i = plan.tiles_i;
  p.tiles_j = plan.tiles_j;
  p.kblocks = plan.kblocks;
  p.splits = plan.splits;
  p.epilogue = kEpiQkvRotary;
  p.ohw = 1;
  p.bias = bqkv;
  p.out = nullptr;
  p.err = device_error_word();
  p.const_a = 1;
  p.rot_cos = cos_table;
  p.rot_sin = sin_table;
  p.rot_pos = positions;
  p.rot_q = q_out;
  p.rot_k = cache_k;
  p.rot_v = cache_v;
  p.rot_hq = static_cast<int>(q_heads);
  p.rot_hkv = static_cast<int>(kv_heads);
  p.rot_d = static_cast<int>(head_dim);
  p.rot_seq = static_cast<int>(seq);
  p.rot_pairs = pairs;
  p.rot_rows = table_rows;
  p.rot_cap = capacity;
  return bf16 ? launch_tc_bn<__nv_bfloat16>(plan.bn, plan.stages, ma, mb, p, plan.splits, as_stream(stream))
              : launch_tc_bn<__half>(plan.bn, plan.stages, ma, mb, p, plan.splits, as_stream(stream));
}

extern "C" dli_status dli_sm100_linear_silu_mul(const void* x, const void* w_glu, void* y, int64_t m,
                                                int64_t inter, int64_t k, dli_dtype dtype, void* stream) {
  const char* name = "linear_silu_mul";
  if (m < 0 || inter <= 0 || k <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad sizes");
  if (dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": bfloat16/float16 only (tcgen05 epilogue)");
  if (m == 0) return ok();
  if (!x || !w_glu || !y) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
  if (!aligned(x, 16) || !aligned(w_glu, 16) || k % 8 != 0)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": 16-byte aligned operands and K % 8 == 0 expected");
  const int64_t rows_w = 2 * ceil_div(inter, 64) * 64;  // gate/up blocks, the last one zero-padded
  if (m <= kSwapRows) {
    const GemmPlan plan = plan_tn_gemm(rows_w, m, k, dtype, true);
    if (!plan.tcgen05) return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": shape not served by tcgen05");
    return run_tn_gemm_tcgen05(w_glu, x, nullptr, y, rows_w, m, k, k, k, inter, kEpiGluT, 0, dtype, plan, nullptr,
                               0, as_stream(stream), true, false, inter);
  }
  const GemmPlan plan = plan_tn_gemm(m, rows_w, k, dtype, false);
  if (!plan.tcgen05 || plan.bn % 128 != 0)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": shape not served by tcgen05");
  return run_tn_gemm_tcgen05(x, w_glu, nullptr, y, m, rows_w, k, k, k, inter, kEpiGlu, 0, dtype, plan, nullptr, 0,
                             as_stream(stream), false, true, inter);
}

extern "C" dli_status dli_sm100_matmul(const void* a, const void* b, void* out, int64_t m, int64_t n,
                                       int64_t k, dli_dtype dtype, void* stream) {
  if (m < 0 || n <= 0 || k <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "matmul: bad sizes");
  if (!is_float_dtype(dtype)) return fail(DLI_ERR_INVALID_ARGUMENT, "matmul expects a float dtype");
  if (m == 0) return ok();
  if (!a || !b || !out) return fail(DLI_ERR_INVALID_ARGUMENT, "matmul: null pointer");
  if (dtype == DLI_DTYPE_F32) {
    dli_status st = DLI_OK;
    if (try_gemm_f32x3(a, b, nullptr, out, m, n, k, n, n, kEpiRowMajor, true, as_stream(stream), &st)) return st;
  }
  // bf16/f16 on tcgen05: A [M,K] K-major, B [K,N] MN-major through 64-column
  // TMA panels (tile width >= 64). Other shapes/alignments take the SIMT kernel.
  GemmPlan plan = plan_tn_gemm(m, n, k, dtype, true);
  if (plan.tcgen05 && n % 8 == 0 && aligned(a, 16) && aligned(b, 16)) {
    if (plan.bn < 64) {
      plan = plan_tn_gemm(m, 64, k, dtype, true);  // the 64-wide plan, N columns masked by TMA/epilogue
      plan.tiles_j = 1;
    }
    return run_tn_gemm_tcgen05(a, b, nullptr, out, m, n, k, k, n, n, kEpiRowMajor, 0, dtype, plan, nullptr, 0,
                               as_stream(stream), false, false, 0, false, true);
  }
  return run_gemm_simt(a, b, nullptr, out, m, n, k, false, dtype, as_stream(stream));
}
