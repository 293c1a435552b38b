// Internal declarations shared by the libamcuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/amc.h"

namespace amc {

// ------------------------------------------------------------------ errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
#define AMC_CUDA(call)                                         \
  do {                                                         \
    cudaError_t _e = (call);                                   \
    if (_e != cudaSuccess) return ::amc::cuda_fail(_e, #call); \
  } while (0)

// Host-side fault injection: AMC_FAULT=alloc|launch|timeout makes the named
// class of operation fail with AMC_ERR_INJECTED before touching the device.
bool fault_injected(const char* what);

size_t dtype_size(int32_t dtype);
bool dtype_valid(int32_t dtype);
bool dtype_float(int32_t dtype);

// ------------------------------------------------------------------ buffers
struct Buffer {
  void* ptr = nullptr;
  int32_t dtype = AMC_F64;
  int64_t nelem = 0;
  bool owned = true;
  int device = 0;
  std::atomic<int> refs{1};
  std::shared_ptr<void> keepalive;  // arena backing for context sub-buffers
};

uint64_t buf_register(Buffer* b);
Buffer* buf_get(uint64_t h);
void buf_retain(uint64_t h);
void buf_release(uint64_t h);
int buf_alloc(int32_t dtype, int64_t nelem, uint64_t* out);

cudaStream_t default_stream();
inline cudaStream_t pick_stream(void* s) { return s ? (cudaStream_t)s : default_stream(); }

// Raise the dynamic shared-memory limit of kernel `fn` to `bytes` on the
// current device, once per device (a function attribute applies to one
// device; `done` holds one bit per device ordinal).
template <typename F>
inline int smem_attr_once(F* fn, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return 0;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  done.fetch_or(bit, std::memory_order_release);
  return 0;
}
int num_sms();

// ------------------------------------------------------------------ device descriptors
struct DLeaf {
  const void* ptr;       // base pointer with the view offset folded in
  int32_t dtype;
  int32_t _pad;
  int64_t strides[AMC_MAX_RANK];  // over the kernel's index space (0 = broadcast)
};

constexpr int kMaxLeaves = 8;

struct DProg {
  int32_t n;
  int32_t all_float;     // every load is f32/f64 and no ICONST: inexact-only evaluation
  int32_t max_depth;     // deepest stack the program reaches
  int32_t _pad;
  amc_insn code[AMC_PROG_MAX];
};

// Element-wise launch: out[i] = store(out_dtype, prog(leaves at i)), i over shape.
struct MapArgs {
  int32_t rank;
  int32_t nleaf;
  int64_t shape[AMC_MAX_RANK];
  int64_t total;
  DLeaf leaf[kMaxLeaves];
  DProg prog;
  void* out;
  int32_t out_dtype;
  int32_t _pad;
};

// Reduction launch: source index space = (kept dims..., reduced dims...) after
// the planner has permuted the reduced axes last and collapsed dims.
struct ReduceArgs {
  int32_t orank, rrank;
  int64_t oshape[AMC_MAX_RANK];   // kept dims (row-major output order)
  int64_t rshape[AMC_MAX_RANK];   // reduced dims (row-major source order)
  int64_t O, R;
  int32_t nleaf;
  int32_t src_dtype;              // dtype of the reduced values (source node)
  DLeaf leaf_o[kMaxLeaves];       // leaf strides over kept dims
  int64_t leaf_r[kMaxLeaves][AMC_MAX_RANK];  // leaf strides over reduced dims
  DProg prog;
  void* out;
  int32_t out_dtype;
  int32_t op;                     // AMC_RED_*
};

int launch_map(const MapArgs& a, cudaStream_t s);

// Fold / scan over axis 0 of x: acc <- round(acc_dtype, prog(acc, x[i])) for
// i = 0..n-1 from acc = init, at every element position (shape, P positions).
// Leaf 0 is init, leaf 1 is x[0] (xstep apart along axis 0).
struct ScanArgs {
  int32_t rank;
  int32_t keep;                   // 1: every accumulator, out (n, shape); 0: the last, out (shape)
  int64_t shape[AMC_MAX_RANK];
  int64_t P, n, xstep;
  DLeaf leaf[2];
  DProg prog;
  void* out;
  int32_t out_dtype;
  int32_t acc_dtype;
};
int launch_scan(const ScanArgs& a, cudaStream_t s);
int launch_reduce(const ReduceArgs& a, cudaStream_t s, void* scratch, size_t scratch_bytes, size_t* scratch_need);
// The column fold (amc_colfold.cu): launched, or AMC_ERR_UNSUPPORTED when the
// reduction is not of its kind (nothing launched, no error recorded).
int launch_colfold(const ReduceArgs& a, cudaStream_t s);
long long colfold_launch_count();

struct PadArgs {
  int32_t rank, mode;
  int64_t oshape[AMC_MAX_RANK];
  int64_t sshape[AMC_MAX_RANK];
  int64_t sstrides[AMC_MAX_RANK];
  int64_t before[AMC_MAX_RANK];
  const void* src; int32_t src_dtype;
  void* out; int32_t out_dtype;
  double value;
  int64_t total;
};
int launch_pad(const PadArgs& a, cudaStream_t s);

struct Im2colArgs {
  int64_t N, C, H, W, OH, OW;
  int32_t KH, KW, SH, SW, PH, PW;
  int64_t sN, sC, sH, sW;
  const void* src; int32_t src_dtype;
  void* out; int32_t out_dtype;
};
int launch_im2col(const Im2colArgs& a, cudaStream_t s);

struct Col2imArgs {
  int64_t N, C, H, W, OH, OW;
  int32_t KH, KW, SH, SW, PH, PW;
  const void* col; int32_t col_dtype;   // contiguous (N, C*KH*KW, OH*OW)
  void* out; int32_t out_dtype;
};
int launch_col2im(const Col2imArgs& a, cudaStream_t s);

struct RouteArgs {
  int32_t rank, axis, is_stack, nsrc;
  int64_t oshape[AMC_MAX_RANK];
  const DLeaf* srcs;         // device array of nsrc source views (strides in source dims)
  const int64_t* extents;    // device array: each source's size along axis (concat)
  void* out; int32_t out_dtype;
  int64_t total;
};
int launch_route(const RouteArgs& a, cudaStream_t s);

// C[M,N] = A[M,K] B[K,N] with arbitrary element strides, double accumulation,
// stored as out_dtype (row-major contiguous output with leading dim N).
struct GemmArgs {
  int64_t M, N, K;
  const void* A; int32_t a_dtype; int64_t sa0, sa1;
  const void* B; int32_t b_dtype; int64_t sb0, sb1;
  void* C; int32_t c_dtype;
  double alpha, beta;            // C = alpha*AB + beta*C (beta=0 ignores C)
};

// GEMM whose result feeds only an element-wise map: the map runs in the
// GEMM's store, with its leaf `leaf` standing for the GEMM result.
struct GemmEpiArgs {
  GemmArgs g;
  MapArgs map;
  int32_t leaf;
  int32_t _pad;
};
int launch_gemm(const GemmArgs& a, cudaStream_t s);
int launch_gemm_epi(const GemmEpiArgs& a, cudaStream_t s);

// Row passes over a row-major X (rows x d, unit stride along d); see
// amc_rowpass.cu.  fwd: p_i = X[i,:] . w stored (alpha/beta, rounded) at
// r[i*sr]; acc: out[k] = sum_i X[i,k] e_i, with e_i = prog(leaves at row i)
// whose leaf e_rleaf is the stored p_i (fwd) or e_i = b[i*sb] (no fwd);
// dot: out = sum_i X[i*ldx] b[i*sb].  Leaf strides[0] is the stride along
// the row index.  partials: scratch of rowpass_scratch_bytes().
struct RowPassArgs {
  int64_t rows;
  int32_t d, x_dtype;
  const void* X; int64_t ldx;
  int32_t fwd, acc, dot, e_rleaf;
  const void* w; int32_t w_dtype; int32_t _p0; int64_t sw;
  void* r; int32_t r_dtype; int32_t _p1; int64_t sr;
  const void* b; int32_t b_dtype; int32_t _p2; int64_t sb;
  int32_t nleaf; int32_t _p3;
  DLeaf leaf[kMaxLeaves];
  DProg prog;
  // The row program in closed form when it is the residual form
  // k * ((c1 * c2) * (p - y)) (k 1 or 2; c1, c2 and y a leaf or a constant,
  // c2 possibly absent; each operation rounded as the program rounds it):
  // set by rowpass_prepare.
  int32_t closed, ck, c_leaf, c2_leaf, y_leaf, c2_used;   // *_leaf -1: the constant
  double c_const, c2_const, y_const;
  // A full sum of (p - y2)^2 over the rows taken in the same pass (the MSE
  // loss's reduction; closed form only): each CTA adds its rows' values into
  // partials[grid * d + CTA]; rsum_y_leaf -1: the constant rsum_y_const.
  int32_t rsum, rsum_y_leaf;
  double rsum_y_const;
  void* out; int32_t out_dtype; int32_t _p4; int64_t sout;
  double alpha, beta;
  double* partials;
};
constexpr int kRowPassMaxD = 1024;
// Contractions at least this large leave k_gemm's sequential order for the
// row passes (elements of A; rows of a transposed GEMV; dot length).
constexpr int64_t kRowPassMinElems = (int64_t)1 << 20;
constexpr int64_t kRowPassMinRows = (int64_t)1 << 14;
constexpr int64_t kRowPassMinDot = (int64_t)1 << 16;
int rowpass_grid(int64_t rows);
size_t rowpass_scratch_bytes(const RowPassArgs& a);
// The row sum's second pass: out = sum of the n partials (fixed order),
// divided by `div` when div != 0 (a mean), stored as out_dtype.
int launch_rowsum_finish(const double* partials, int n, void* out, int out_dtype, double div, cudaStream_t s);
// The number of CTAs that write partial rows for `a`.
int rowpass_ctas(const RowPassArgs& a);
// Whether the GEMV pair `a` runs the TMA pipeline (contiguous rows).
bool rowpass_pair_tma(const RowPassArgs& a);
int rowpass_launches(const RowPassArgs& a);
int launch_rowpass(const RowPassArgs& a, cudaStream_t s);
// Once per planned launch: finds a closed form of the row program.
void rowpass_prepare(RowPassArgs& a);
// GEMM dispatch with the row passes: scratch of gemm_scratch_bytes(g)
// (0: none needed), launches per execute.
bool gemm_as_rowpass(const GemmArgs& g, RowPassArgs& r);
size_t gemm_scratch_bytes(const GemmArgs& g);
int gemm_launches(const GemmArgs& g);
int launch_gemm_scratch(const GemmArgs& g, void* scratch, cudaStream_t s);

struct AttnArgs {
  int64_t blocks;
  int32_t n, dk, dv, dtype;
  const void* Q; int64_t qb, q0, q1;
  const void* K; int64_t kb, k0, k1;
  const void* V; int64_t vb, v0, v1;
  void* O;                        // contiguous (blocks, n, dv)
  double scale;
};
int launch_attention_generic(const AttnArgs& a, cudaStream_t s);
// Tensor-core attention forward for contiguous f32 (blocks, n, 64) operands,
// n a multiple of 128; sets *handled = false (and launches nothing) otherwise.
int attention_fwd_tc(const float* Q, const float* K, const float* V, float* O, float* lse, long long blocks, int n,
                     int dk, int dv, float scale, cudaStream_t s, bool* handled);
// Tensor-core attention backward for the same operands (n a multiple of 128);
// sets *handled = false (and launches nothing) for other shapes.
int attention_bwd_tc(const float* Q, const float* K, const float* V, const float* O, const float* dO,
                     const float* lse, float* dQ, float* dK, float* dV, long long blocks, int n, int dk, int dv,
                     float scale, cudaStream_t s, bool* handled);

// Windowed FIR (the polyphase filter-bank reduction).
struct FirArgs {
  const float* x; int64_t batch, x_bstride, frames, hop;
  int32_t taps, branches;
  int64_t x_tstride;              // stride between taps (== branches for the filter bank)
  const float* h; int64_t h_tstride;   // h[t*h_tstride + m]
  float* out; int64_t o_bstride, o_fstride;  // out[b*o_bstride + f*o_fstride + m]
};
bool fir_supported(const FirArgs& a);
int launch_fir(const FirArgs& a, cudaStream_t s);
int fir_launches(const FirArgs& a);
int fir_check_error();   // reads and clears the device-side wait-timeout flag
int attention_check_error();
int attention_bwd_check_error();
int conv_check_error();
int rowpass_check_error();
int colfold_check_error();
int dist_check_error();
int device_check_errors();  // all kernels' bounded-wait flags

}  // namespace amc
