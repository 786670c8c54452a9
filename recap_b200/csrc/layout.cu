// Layout gather fused with block pooling and the per-call closure statistics of K.
//
// One pass over the native-order Q, K and V of a layer call, one CTA per 128-token block:
//  * reorders the tokens into [Hilbert-ordered video | text] (Layout.reorder,
//    recap/sparse/layout.py:86-90), writing Q and K as [banks, S_pad, D] and V
//    transposed as [banks, D, S_pad] (the K-major operand layout of P V);
//  * sums each block over its video tokens in fp32 and divides by the token count
//    (pool_blocks, recap/sparse/pooling.py:10-34): fp32 means plus the bf16 copies the
//    coarse tail reads;
//  * writes the block-centred video keys k - kbar, transposed and rounded to bf16, as
//    the K-major B operand of the C_vk GEMM (recap/kernels/closure_stats.py:27-94);
//  * with a basis U and 0 < rank < D, the rank-folded per-block key variances in U
//    (rotated_leaf_moments_triton + fold_rank, recap/kernels/closure_stats.py:96-189,
//    recap/sparse/closure.py:96-104): the leading `rank` columns are the two-pass
//    population variances of K U[:, c]; every other column is their mean, which for an
//    orthonormal U equals (trace of the block covariance - the leading variances) /
//    (D - rank), so only K U[:, :rank] is formed.
//  * the norm bounds the softmax kernels use to skip their running-max work: the
//    largest |k| over each block's tokens and |bf16(kbar)| of each video block.
// Rows past S (up to S_pad) are written as zeros.  HBM-bound.
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxRank = 8;

__device__ __forceinline__ void add8(float (&acc)[8], const uint4& w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(h[e]);
    acc[2 * e] += f.x;
    acc[2 * e + 1] += f.y;
  }
}

// Four 8x8 bf16 matrices from shared memory, each lane addressing one 16-byte row.
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// The same, each matrix transposed on the way (thread i receives column i / 4, rows
// 2 (i % 4) and 2 (i % 4) + 1).
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// 16-byte asynchronous copy from global to shared memory through L2 only; src_bytes = 0
// writes sixteen zero bytes and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// d += a * b for one 16x8x16 bf16 tile with fp32 accumulation (warp-wide).
__device__ __forceinline__ void mma_m16n8k16_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Staged 128 x D bf16 tiles: rows of D * 2 bytes, the 16-byte chunks of row r stored at
// chunk ^ ((r / 8) mod (D / 8)).  One chunk of eight rows spaced eight apart lies in eight
// different bank groups, and lanes that read a row see a permutation of its chunks.
template <int D>
__device__ __forceinline__ uint32_t stage_off(int r, int chunk) {
  constexpr int CPR = D / 8;
  return static_cast<uint32_t>(r * (D * 2) + ((chunk ^ ((r >> 3) & (CPR - 1))) << 4));
}
template <int D>
__device__ __forceinline__ __nv_bfloat16 stage_elem(const uint8_t* tile, int r, int d) {
  return *reinterpret_cast<const __nv_bfloat16*>(tile + stage_off<D>(r, d >> 3) + (d & 7) * 2);
}

template <int D>
struct GatherSmem {
  static constexpr int kV = 0;
  static constexpr int kK = kV + 128 * D * 2;
  static constexpr int kRed = kK + 128 * D * 2;              // [RPP][D] fp32
  static constexpr int kMean = kRed + 32 * D * 4;            // [D] fp32 key means
  // leading basis columns as mma.m16n8k16 B fragments, U = hi + mid + lo in bf16:
  // [part][k-step][lane][4] bf16
  static constexpr int kUf = kMean + D * 4;
  static constexpr int kStat = kUf + 3 * (D / 16) * 32 * 8;  // [2*kMaxRank + 1]
  static constexpr int kTotal = kStat + 64 * 4;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 2) gather_kernel(const GatherArgs a) {
  using L = GatherSmem<D>;
  constexpr int CPR = D / 8;              // 16-byte chunks per row
  constexpr int RPP = kThreads / CPR;     // rows per pass
  constexpr int PASSES = 128 / RPP;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* vtile = smem + L::kV;
  uint8_t* ktile = smem + L::kK;
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* kmean_s = reinterpret_cast<float*>(smem + L::kMean);
  __nv_bfloat16* ufrag = reinterpret_cast<__nv_bfloat16*>(smem + L::kUf);
  float* stat = reinterpret_cast<float*>(smem + L::kStat);

  const int blk = blockIdx.x;
  const int bank = blockIdx.y;
  const int bi = bank / a.heads;
  const int hi = bank - bi * a.heads;
  const int tid = threadIdx.x;
  const int ch = tid % CPR;
  const int rsub = tid / CPR;
  const int row0 = blk * 128;
  const int video_rows = min(128, a.n_video - row0);  // <= 0 for text-only blocks
  const bool need_k_tile = (a.kct != nullptr || a.variance != nullptr) && video_rows > 0;

  // The variance pass's leading basis columns U[d][0 .. rank) (zero past the rank), staged
  // now so that their loads overlap the gathers (ufrag is read only after later barriers).
  // Each value is split into three bf16 parts, hi + mid + lo, whose sum is the fp32 value
  // to within 2^-24 relative: the tensor-core products of bf16 keys with each part are
  // exact, so the rotation keeps fp32 accuracy.  Element (d, c) goes where lane 4c + t of
  // an m16n8k16 B fragment holds it: k-step d / 16, t = (d % 8) / 2, register (d % 16) / 8.
  if (a.variance != nullptr && blk < a.nB && video_rows > 0 && tid < D) {
    const float* U = a.basis + (static_cast<size_t>(bank) * D + tid) * D;
    const int ks = tid >> 4;
    const int w16 = tid & 15;
    const int slot = (w16 >> 3) * 2 + (w16 & 1);
    const int t = (w16 & 7) >> 1;
#pragma unroll
    for (int c = 0; c < kMaxRank; ++c) {
      const float u = c < a.rank ? U[c] : 0.f;
      const __nv_bfloat16 hi = __float2bfloat16_rn(u);
      const float r1 = u - __bfloat162float(hi);
      const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
      const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
      const int lane_c = c * 4 + t;
      ufrag[((0 * (D / 16) + ks) * 32 + lane_c) * 4 + slot] = hi;
      ufrag[((1 * (D / 16) + ks) * 32 + lane_c) * 4 + slot] = mid;
      ufrag[((2 * (D / 16) + ks) * 32 + lane_c) * 4 + slot] = lo;
    }
  }

  // Native rows of this thread's PASSES rows; each tensor's PASSES row chunks then go
  // out in one burst of independent loads (Q to registers, K and V by asynchronous copies
  // below), so the pass waits on one gather latency rather than one per row.
  int nat[PASSES];
#pragma unroll
  for (int p = 0; p < PASSES; ++p) {
    const int r = row0 + p * RPP + rsub;
    int n = -1;
    if (r < a.S) {
      n = a.src_row[r];
      if (n < 0 || n >= a.S) n = -1;  // a corrupt index reads nothing out of bounds
    }
    nat[p] = n;
  }
  // Address of this thread's chunk of native token n of tensor t: in the one source, or in
  // the token shard of the rank that holds n.
  auto row_src = [&](int t, int n) -> const __nv_bfloat16* {
    const int64_t off = bi * a.stride_b[t] + hi * a.stride_h[t] + ch * 8;
    if (a.n_ranks > 1) {
      const int q = n / a.tokens_per_rank;
      return a.rank_src[q][t] + off + static_cast<int64_t>(n - q * a.tokens_per_rank) * a.stride_s[t];
    }
    return a.src[t] + off + static_cast<int64_t>(n) * a.stride_s[t];
  };
  auto load_rows = [&](int t, uint4 (&v)[PASSES]) {
    if (a.src[t] == nullptr) return;
#pragma unroll
    for (int p = 0; p < PASSES; ++p) v[p] = nat[p] >= 0 ? ld_stream_v4(row_src(t, nat[p])) : make_uint4(0, 0, 0, 0);
  };
  float knorm2 = 0.f;  // largest |k|^2 over this thread's rows
  auto process = [&](int t, const uint4 (&v)[PASSES]) {
    if (a.src[t] == nullptr) return;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int p = 0; p < PASSES; ++p) {
      const int rl = p * RPP + rsub;
      const int r = row0 + rl;
      const uint4 val = v[p];
      if (t == 0 && a.qr) {
        *reinterpret_cast<uint4*>(a.qr + (static_cast<size_t>(bank) * a.S_pad + r) * D + ch * 8) = val;
      } else if (t == 1 && a.kr) {
        *reinterpret_cast<uint4*>(a.kr + (static_cast<size_t>(bank) * a.S_pad + r) * D + ch * 8) = val;
      }
      if (rl < video_rows) add8(acc, val);
      if (t == 1 && a.k_norm_max) {
        // |k|^2 of row rl: this lane's 8 dims, summed over the 16 lanes of the row
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&val);
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
        }
#pragma unroll
        for (int o = CPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        knorm2 = fmaxf(knorm2, ss);
      }
    }
    const bool want_mean = blk < a.nB && (a.mean[t] != nullptr || (t == 1 && (need_k_tile || a.k_mean_norm)));
    if (want_mean) {
#pragma unroll
      for (int e = 0; e < 8; ++e) red[rsub * D + ch * 8 + e] = acc[e];
      __syncthreads();
      if (tid < D) {
        float sum = 0.f;
#pragma unroll 4
        for (int g = 0; g < RPP; ++g) sum += red[g * D + tid];
        const float m = sum / static_cast<float>(video_rows);
        if (t == 1) {
          kmean_s[tid] = m;
          if (a.k_mean_norm) {
            // |bf16(kbar)|^2 over the D columns (threads 0 .. D-1, whole warps)
            const float mb = __bfloat162float(__float2bfloat16_rn(m));
            float q = mb * mb;
            for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            if ((tid & 31) == 0) stat[32 + (tid >> 5)] = q;
          }
        }
        if (a.mean[t]) a.mean[t][(static_cast<size_t>(bank) * a.nB + blk) * D + tid] = m;
        if (t == 1 && a.kmean_bf16)
          a.kmean_bf16[(static_cast<size_t>(bank) * a.nB_pad + blk) * D + tid] = __float2bfloat16_rn(m);
        if (t == 2 && a.vmean_t_bf16)
          a.vmean_t_bf16[(static_cast<size_t>(bank) * D + tid) * a.nB_pad + blk] = __float2bfloat16_rn(m);
      }
      __syncthreads();
      if (t == 1 && a.k_mean_norm && tid == 0) {
        float q = 0.f;
        for (int w = 0; w < D / 32; ++w) q += stat[32 + w];
        a.k_mean_norm[static_cast<size_t>(bank) * a.nB + blk] = sqrtf(q);
      }
    }
  };
  {
    // K and V go straight into their staged tiles by asynchronous copies (no registers),
    // so the loads of all three tensors are in flight at once; Q comes to registers and
    // is stored from there.  K and V are read back from shared memory for their stores,
    // pools and norms.
    auto copy_rows = [&](int t, uint8_t* tile) {
      if (a.src[t] == nullptr) return;
#pragma unroll
      for (int p = 0; p < PASSES; ++p) {
        const bool in = nat[p] >= 0;
        cp_async16(smem_u32(tile + stage_off<D>(p * RPP + rsub, ch)), row_src(t, in ? nat[p] : 0), in ? 16u : 0u);
      }
    };
    auto read_rows = [&](const uint8_t* tile, uint4 (&v)[PASSES]) {
#pragma unroll
      for (int p = 0; p < PASSES; ++p) v[p] = *reinterpret_cast<const uint4*>(tile + stage_off<D>(p * RPP + rsub, ch));
    };
    copy_rows(1, ktile);
    copy_rows(2, vtile);
    cp_async_commit();
    uint4 va[PASSES];
    load_rows(0, va);
    process(0, va);
    cp_async_wait_all();
    __syncthreads();  // every thread's copies have landed
    read_rows(ktile, va);
    process(1, va);
    read_rows(vtile, va);
    process(2, va);
  }
  if (a.k_norm_max) {
    // block maximum of the row norms: warp maxima, then one thread
    float m2 = knorm2;
    for (int o = 16; o > 0; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
    if ((tid & 31) == 0) stat[48 + (tid >> 5)] = m2;
    __syncthreads();
    if (tid == 0) {
      float mm = 0.f;
      for (int w = 0; w < kThreads / 32; ++w) mm = fmaxf(mm, stat[48 + w]);
      a.k_norm_max[static_cast<size_t>(bank) * (a.S_pad / 128) + blk] = sqrtf(mm);
    }
  }

  __syncthreads();  // the staged V and K tiles are complete before anyone reads them back
  // Transposed stores (V^T and the centred K^T): for each head dimension d this block owns
  // 128 contiguous bf16 of row d.  A warp takes a tile of 32 tokens x 8 dimensions with one
  // transposing ldmatrix: lane (j, q) addresses token 8(q/2) + 2j + q%2 of the tile, so that
  // thread (dl, tq) receives dimension dl of tokens 8tq .. 8tq + 7 in order, one 16-byte
  // store; a warp instruction writes eight 64-byte runs.
  {
    const int lane = tid & 31;
    const int warp = tid >> 5;
    constexpr int kWarps = kThreads / 32;
    constexpr int kTiles = 4 * (D / 8);  // 4 token groups x D/8 dimension blocks
    const int tok_in = 8 * ((lane & 7) >> 1) + 2 * (lane >> 3) + (lane & 1);
    const int dl = lane >> 2;
    const int tq = lane & 3;
    if (a.vt != nullptr && a.src[2] != nullptr) {
      for (int tile = warp; tile < kTiles; tile += kWarps) {
        const int tg = tile & 3;
        const int db = tile >> 2;
        uint32_t r[4];
        ldmatrix_x4_trans(r, smem_u32(vtile + stage_off<D>(32 * tg + tok_in, db)));
        *reinterpret_cast<uint4*>(a.vt + (static_cast<size_t>(bank) * D + 8 * db + dl) * a.S_pad + row0 + 32 * tg +
                                  8 * tq) = make_uint4(r[0], r[1], r[2], r[3]);
      }
    }
    if (a.kct != nullptr) {
      // centred video keys, bf16; zero outside the video tokens
      for (int tile = warp; tile < kTiles; tile += kWarps) {
        const int tg = tile & 3;
        const int db = tile >> 2;
        const int d = 8 * db + dl;
        const float m = video_rows > 0 ? kmean_s[d] : 0.f;
        uint32_t r[4];
        ldmatrix_x4_trans(r, smem_u32(ktile + stage_off<D>(32 * tg + tok_in, db)));
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t0 = 32 * tg + 8 * tq + 2 * e;
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[e]));
          const float x0 = t0 < video_rows ? f.x - m : 0.f;
          const float x1 = t0 + 1 < video_rows ? f.y - m : 0.f;
          const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
          r[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(a.kct + (static_cast<size_t>(bank) * D + d) * a.S_pad + row0 + 32 * tg + 8 * tq) =
            make_uint4(r[0], r[1], r[2], r[3]);
      }
    }
  }

  if (a.variance != nullptr && blk < a.nB && video_rows > 0) {
    const int rank = a.rank;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // Rotated values of the leading columns, rot[r][c] = sum_d k[r][d] U[d][c], on the tensor
    // cores: warp w takes the sixteen rows 8m + w (m = 0 .. 15; the stride makes the eight
    // rows of each ldmatrix phase fall in eight different swizzle chunks, so the loads are
    // free of bank conflicts) and one m16n8k16 MMA per k-step and part of U.  Thread (g, t)
    // ends with rows 8g + w and 8(g + 8) + w, columns 2t and 2t + 1.
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int mrow = ((lane >> 3) & 1) * 8 + (lane & 7);  // ldmatrix row of this lane's address
      const int kc = lane >> 4;                             // which 8-column half of the k-step
      const uint2* bf = reinterpret_cast<const uint2*>(ufrag);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t af[4];
        ldmatrix_x4(af, smem_u32(ktile + stage_off<D>(8 * mrow + warp, 2 * ks + kc)));
#pragma unroll
        for (int part = 0; part < 3; ++part) {
          const uint2 b = bf[(part * (D / 16) + ks) * 32 + lane];
          mma_m16n8k16_bf16(acc, af, b.x, b.y);
        }
      }
    }
    const int g = lane >> 2;
    const int t = lane & 3;
    const bool v0 = 8 * g + warp < video_rows;
    const bool v1 = 8 * (g + 8) + warp < video_rows;
    // The trace of the block covariance, sum_d sum_r (k[r][d] - m_d)^2: thread (part, pair)
    // takes dimensions 2 pair and 2 pair + 1 over its share of the rows.
    float tr;
    {
      constexpr int kPairs = D / 2;
      constexpr int kParts = kThreads / kPairs;
      constexpr int kRowsPer = 128 / kParts;
      const int pr = tid % kPairs;
      const int part = tid / kPairs;
      const float m0 = kmean_s[2 * pr];
      const float m1 = kmean_s[2 * pr + 1];
      const int r0 = part * kRowsPer;
      const int r1 = min(r0 + kRowsPer, video_rows);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
      for (int rr = r0; rr < r1; ++rr) {
        const float2 f = __bfloat1622float2(
            *reinterpret_cast<const __nv_bfloat162*>(ktile + stage_off<D>(rr, pr >> 2) + (pr & 3) * 4));
        const float x0 = f.x - m0;
        const float x1 = f.y - m1;
        s0 = fmaf(x0, x0, s0);
        s1 = fmaf(x1, x1, s1);
      }
      tr = s0 + s1;
    }
    for (int o = 16; o > 0; o >>= 1) tr += __shfl_xor_sync(0xffffffffu, tr, o);
    // Two-pass population variances of the rotated columns: column sums over the video rows
    // (lanes of equal t, then the eight warps), the means, then the squared deviations.
    float* colsum = red + 64;   // [8 warps][kMaxRank]; red (the pooling scratch) is free since the
                                // barrier before the transposed stores
    float* colsq = red + 128;   // [8 warps][kMaxRank]
    float cs0 = (v0 ? acc[0] : 0.f) + (v1 ? acc[2] : 0.f);
    float cs1 = (v0 ? acc[1] : 0.f) + (v1 ? acc[3] : 0.f);
    for (int o = 4; o < 32; o <<= 1) {
      cs0 += __shfl_xor_sync(0xffffffffu, cs0, o);
      cs1 += __shfl_xor_sync(0xffffffffu, cs1, o);
    }
    if (lane == 0) red[warp] = tr;
    if (lane < 4) {
      colsum[warp * kMaxRank + 2 * t] = cs0;
      colsum[warp * kMaxRank + 2 * t + 1] = cs1;
    }
    __syncthreads();
    const float inv_n = 1.f / static_cast<float>(video_rows);
    float mc0 = 0.f, mc1 = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      mc0 += colsum[w * kMaxRank + 2 * t];
      mc1 += colsum[w * kMaxRank + 2 * t + 1];
    }
    mc0 *= inv_n;
    mc1 *= inv_n;
    float q0 = 0.f, q1 = 0.f;
    if (v0) {
      const float x0 = acc[0] - mc0, x1 = acc[1] - mc1;
      q0 = x0 * x0;
      q1 = x1 * x1;
    }
    if (v1) {
      const float x0 = acc[2] - mc0, x1 = acc[3] - mc1;
      q0 = fmaf(x0, x0, q0);
      q1 = fmaf(x1, x1, q1);
    }
    for (int o = 4; o < 32; o <<= 1) {
      q0 += __shfl_xor_sync(0xffffffffu, q0, o);
      q1 += __shfl_xor_sync(0xffffffffu, q1, o);
    }
    if (lane < 4) {
      colsq[warp * kMaxRank + 2 * t] = q0;
      colsq[warp * kMaxRank + 2 * t + 1] = q1;
    }
    __syncthreads();
    if (tid < D) {
      float lead = 0.f;
      float v = 0.f;
      for (int c = 0; c < rank; ++c) {
        float q = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) q += colsq[w * kMaxRank + c];
        q = fmaxf(q * inv_n, 0.f);
        lead += q;
        if (c == tid) v = q;
      }
      if (tid >= rank) {
        float total = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) total += red[w];
        total *= inv_n;
        v = fmaxf(total - lead, 0.f) / static_cast<float>(D - rank);
      }
      a.variance[(static_cast<size_t>(bank) * a.nB + blk) * D + tid] = v;
      if (a.variance_bf16)
        a.variance_bf16[(static_cast<size_t>(bank) * a.nB_pad + blk) * D + tid] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace

int launch_gather(const GatherArgs& a, cudaStream_t s) {
  if (a.S_pad % 128 || a.S > a.S_pad || a.n_video > a.S || a.n_video <= 0) return kErrShape;
  if (a.variance != nullptr && (a.basis == nullptr || a.rank <= 0 || a.rank >= a.D || a.rank > kMaxRank))
    return kErrShape;
  dim3 grid(a.S_pad / 128, a.batch * a.heads);
  if (a.D == 128) {
    const int smem = GatherSmem<128>::kTotal;
    cudaFuncSetAttribute(gather_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    gather_kernel<128><<<grid, kThreads, smem, s>>>(a);
  } else if (a.D == 64) {
    const int smem = GatherSmem<64>::kTotal;
    cudaFuncSetAttribute(gather_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    gather_kernel<64><<<grid, kThreads, smem, s>>>(a);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int gather_max_rank() { return kMaxRank; }

}  // namespace recap
