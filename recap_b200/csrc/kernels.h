// Internal launch interface of the CUDA kernels (host side of each .cu file).
// The public C ABI lives in include/recap_b200.h and recap_b200/csrc/capi.cu.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace recap {

// Largest number of ranks whose buffers one launch reads from or writes to directly
// (the token shards of a sequence-parallel layer, over NVLink peer mappings).
constexpr int kMaxRanks = 8;

// Host-side status codes (the C ABI returns them).
enum : int {
  kOk = 0,
  kErrShape = 1,    // bad shape, stride or alignment
  kErrLaunch = 2,   // CUDA launch or API failure
  kErrDevice = 3,   // a kernel reported a device-side timeout (see the status word)
  kErrUnsupported = 4,
  kErrScratchLimit = 5,  // larger than the fixed scratch of a no-allocation entry point
};

// ------------------------------------------------------------------ layout gather + pooling
struct GatherArgs {
  int batch, heads, S, S_pad, D, n_video, nB, nB_pad;
  const __nv_bfloat16* src[3];  // q, k, v in native order, [batch, heads, S, D] with strides
  int64_t stride_b[3], stride_h[3], stride_s[3];  // elements; D is contiguous
  const int* src_row;           // [S] native token index of reordered row r
  __nv_bfloat16* qr;            // [banks, S_pad, D] reordered Q (nullable)
  __nv_bfloat16* kr;            // [banks, S_pad, D] reordered K (nullable)
  __nv_bfloat16* vt;            // [banks, D, S_pad] reordered V, transposed (nullable)
  float* mean[3];               // [banks, nB, D] block means over video tokens (nullable each)
  __nv_bfloat16* kmean_bf16;    // [banks, nB_pad, D] (nullable)
  __nv_bfloat16* vmean_t_bf16;  // [banks, D, nB_pad] (nullable)
  __nv_bfloat16* kct;           // [banks, D, S_pad] block-centred video keys, transposed (nullable)
  const float* basis;           // [banks, D, D] fp32 (with variance)
  int rank;                     // 0 < rank < D, rank <= gather_max_rank()
  float* variance;              // [banks, nB, D] rank-folded per-block variance in the basis (nullable)
  __nv_bfloat16* variance_bf16; // [banks, nB_pad, D] (nullable)
  float* k_norm_max;            // [banks, NB] largest |k| over the tokens of each block (nullable)
  float* k_mean_norm;           // [banks, nB] |bf16(kbar)| of each video block (nullable)
  // n_ranks > 1: native token n is row n - q tokens_per_rank of rank q = n / tokens_per_rank,
  // whose tensor t starts at rank_src[q][t] (same strides); src[t] is then rank_src[0][t]
  int n_ranks, tokens_per_rank;
  const __nv_bfloat16* rank_src[kMaxRanks][3];
};
int launch_gather(const GatherArgs& a, cudaStream_t s);
int gather_max_rank();

// ------------------------------------------------------------------ sequence-to-head exchange
struct PushArgs {
  int tokens, heads, heads_per_rank, D;  // this rank's tokens; heads of the layer
  int64_t token0;                        // this rank's first token (its rows in the receive buffers)
  const __nv_bfloat16* src;              // [tokens, 3, heads, D] this rank's projections
  __nv_bfloat16* dst[kMaxRanks];         // [S, 3, heads_per_rank, D] receive buffer of each rank
};
int launch_push(const PushArgs& a, cudaStream_t s);

struct ScatterArgs {
  int banks, S, D, tokens_per_rank;
  int64_t bank_stride, row_stride;     // elements, in every destination
  const __nv_bfloat16* src;            // [banks, S, D]
  __nv_bfloat16* dst[kMaxRanks];       // token shard of each rank
};
int launch_scatter(const ScatterArgs& a, cudaStream_t s);

// ------------------------------------------------------------------ C_vk on tensor cores
struct CvkArgs {
  int banks, n_video, video_steps;  // video_steps = ceil(n_video / 64)
  float* partial;                   // [banks, cvk_chunks, D, D]
  int* status;
};
struct CvkLaunch {
  int D;
  CUtensorMap tm_vt, tm_kct;
  CvkArgs args;
};
int cvk_chunks(int n_video);
int launch_cvk(const CvkLaunch& L, cudaStream_t s);
int launch_moments_reduce(const float* ws, int banks, int nchunks, int D, float inv_n, float* out,
                          __nv_bfloat16* out_bf16, cudaStream_t s);

// ------------------------------------------------------------------ selection
struct SelectArgs {
  int banks, nB, D, keep, n_video, block_size;
  float scale;
  const float* qmean;  // [banks, nB, D]
  const float* kmean;  // [banks, nB, D]
  uint8_t* partition;  // [banks, nB, nB] out
};
int launch_select(const SelectArgs& a, cudaStream_t s);

struct OverlapArgs {
  int64_t n;             // elements of each mask
  const uint8_t* a;      // new partition
  const uint8_t* b;      // old partition
  long long* out;        // [2]: sum(a & b), sum(a)
};
int launch_overlap(const OverlapArgs& a, cudaStream_t s);

struct KernelMaskArgs {
  int banks, nB, NB, dense_start;
  const uint8_t* partition;  // [banks, nB, nB]
  uint8_t* mask;             // [banks, NB, NB]
};
int launch_kernel_mask(const KernelMaskArgs& a, cudaStream_t s);

// ------------------------------------------------------------------ closure statistics
struct ClosureArgs {
  int banks, S_pad, D, n_video, nB, nB_pad, rank;
  const __nv_bfloat16* kr;   // [banks, S_pad, D]
  const __nv_bfloat16* vt;   // [banks, D, S_pad]
  const float* kmean;        // [banks, nB, D]
  const float* basis;        // [banks, D, D] fp32, columns = basis vectors (nullable: skip variance)
  float* scatter;            // [banks, D, D] pooled within-block key scatter (nullable: skip)
  float* cvk;                // [banks, D, D] pooled value-key covariance C_vk (nullable: skip)
  __nv_bfloat16* cvk_bf16;   // [banks, D, D] (nullable)
  float* variance;           // [banks, nB, D] per-block variance in the basis, rank-folded
  __nv_bfloat16* variance_bf16;  // [banks, nB_pad, D] (nullable)
  float* workspace;          // partial sums, see closure_workspace_floats()
};
int64_t closure_workspace_floats(int banks, int D, int nB);
int launch_closure_moments(const ClosureArgs& a, cudaStream_t s);   // scatter and/or C_vk
int launch_closure_variance(const ClosureArgs& a, cudaStream_t s);  // per-block variance

struct BasisPrepArgs {
  int banks, D;
  const float* basis;        // [banks, D, D]
  __nv_bfloat16* basis_t;    // [banks, D, D] out: basis_t[n][k] = basis[k][n], bf16
};
int launch_basis_prep(const BasisPrepArgs& a, cudaStream_t s);

// ------------------------------------------------------------------ coarse tail
struct CoarseArgs {
  int banks, S_pad, D, nB, nB_pad, rows, n_video;
  float scale, theta;
  int rank;                      // w is folded at this rank (columns >= rank equal); 0: not folded
  const uint8_t* partition;      // [banks, nB, nB]
  const float* k_mean_norm;      // [banks, nB] |bf16(kbar)| (nullable: exact maxima every tile)
  const float* counts_log;       // [nB] ln(tokens per video block)
  const float* old_lse;          // [banks, rows] coarse LSE at the last refresh (nullable)
  __nv_bfloat16* out;            // [banks, rows, D] coarse O + gate * drift (bf16)
  float* lse;                    // [banks, rows]
  float* center_partial;         // [banks, rows/128] sum of (lse - old_lse) per query block
  int* status;
};
struct CoarseLaunch {
  int D;
  CUtensorMap tm_q, tm_basis_t, tm_cvk, tm_kmean, tm_var, tm_vmean_t;
  CoarseArgs args;
};
int launch_coarse(const CoarseLaunch& L, cudaStream_t s);

struct CenterArgs {
  int banks, nqb, rows;
  const float* partial;   // [banks, nqb]
  float* center;          // [banks]
};
int launch_center(const CenterArgs& a, cudaStream_t s);

// ------------------------------------------------------------------ FMHA
struct FmhaArgs {
  int banks, S, S_pad, NB, nB, dense_start, rows;
  int all_blocks;          // 1: every key block (dense attention)
  // 1 (with all_blocks): every key block, the partition's kept blocks first; each row's
  // output and LSE over the kept blocks alone go to head_o / head_lse on the way
  int refresh;
  __nv_bfloat16* head_o;   // [banks, S, D] reordered (refresh)
  float* head_lse;         // [banks, S] reordered (refresh)
  float scale_log2;        // softmax scale * log2(e)
  const uint8_t* partition;  // [banks, nB, nB]
  const float* k_norm_max;   // [banks, NB] largest |k| per key block (nullable: always exact maxima)
  int epilogue;            // 0: O and LSE; 1: corrected merge
  const int* out_pos;      // [S] output row of reordered row r (nullptr: r)
  __nv_bfloat16* o;        // [banks, S, D]
  float* lse;              // [banks, S] (nullable)
  const __nv_bfloat16* go; // [banks, rows, D] coarse tail output
  const float* gl;         // [banks, rows] coarse tail LSE
  const __half* det;       // [banks, rows, D] refinement of the tail value
  const float* dl;         // [banks, rows] refinement of the tail log-mass
  const float* ogl;        // [banks, rows] coarse LSE at the refresh
  const float* center;     // [banks]
  int tma_epilogue;        // 1: tm_go / tm_det describe go / det (epilogue 1 with video rows)
  // Output rows: bank b, native position n at o + b o_bank_stride + n o_row_stride (elements;
  // S D and D for a [banks, S, D] output).  n_ranks > 1: at o_rank[q] + b o_bank_stride +
  // (n - q tokens_per_rank) o_row_stride with q = n / tokens_per_rank (token shards of ranks)
  int64_t o_bank_stride, o_row_stride;
  int n_ranks, tokens_per_rank;
  __nv_bfloat16* o_rank[kMaxRanks];
  const __nv_bfloat16* q;  // [banks, S_pad, D] reordered Q (the tiles tm_q reads; L2 prefetch)
  int num_sms;             // SMs of the device: the CTA that follows this one on its SM
  int* status;
};
struct FmhaLaunch {
  int D;
  CUtensorMap tm_q, tm_k, tm_vt;
  CUtensorMap tm_go, tm_det;  // [banks * rows, D] coarse output / refinement, 2-byte elements
  FmhaArgs args;
};
int launch_fmha(const FmhaLaunch& L, cudaStream_t s);
// out[i] = exp2_poly2(in[i]) (the softmax's FP32-pipe exponential)
int launch_exp2_check(const float* in, float* out, int n, cudaStream_t s);
// one bounded mbarrier wait that runs out (status word, abort flag); see selftest.cu
int launch_wait_selftest(int* status, long long limit_ns, long long* result, cudaStream_t s);

// ------------------------------------------------------------------ refresh
struct RefreshArgs {
  int banks, S, D, rows, video_offset;
  const __nv_bfloat16* full_o;  // [banks, S, D] dense O, native order
  const float* full_lse;        // [banks, S] dense LSE, native order
  const __nv_bfloat16* head_o;  // [banks, S, D] head O, reordered
  const float* head_lse;        // [banks, S]
  const __nv_bfloat16* go;      // [banks, rows, D]
  const float* gl;              // [banks, rows]
  const int* perm;              // [>= rows] reordered video position -> native video index
  __half* det;                  // [banks, rows, D] in/out
  float* dl;                    // [banks, rows] in/out
  int validate;                 // score the old refinement first
  const float* ogl;             // [banks, rows] drift reference (nullable: no drift weight)
  const float* center;          // [banks] (with ogl)
  float* partials;              // [n_cta, 2] per-CTA validation sums (validate)
  float* stats;                 // [2] out (validate)
};
int refresh_partials_count(int banks, int rows);
int launch_refresh(const RefreshArgs& a, cudaStream_t s);
// same, with the validation partials in a static device array (no caller scratch)
int launch_refresh_noalloc(RefreshArgs a, cudaStream_t s);

// ------------------------------------------------------------------ tensor maps
// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box = 64 columns x box_rows,
// 128-byte swizzle.  Returns kOk or an error code.
int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                   uint32_t box_rows);

}  // namespace recap
