// Ordered sum of a small element program over one reduced axis whose outputs
// are adjacent in memory: the "column fold" (realization.scm:1309-1388, the
// ordered reduction, with the element program of realization.scm:876-997
// fused in).
//
//   out[o] = fold over r = 0 .. R-1, in that order, of v(o, r)
//
// where every leaf of v is read at ptr + o + r * pitch (elements): the
// outputs are the contiguous axis and the reduced axis is strided.  Config 1
// (sum over axis 1 of x^2 + y on the step-2 slice of a transposed 1024 x 1024
// reshape) is of this kind.
//
// Program-specialised evaluation.  The host turns the element program into
// one closed form
//     v = A,   v = A op1 B,   v = (A op1 B) op2 C   or   v = C op2 (A op1 B)
// with op in {+, -, *} and A, B, C each a leaf or a constant, and the kernel
// evaluates it branch-free on warp-uniform selectors instead of interpreting
// the instruction stream.  Values and rounding are those of the generic
// evaluators: doubles for float programs (rounded to f32 after every
// operation of an f32 program, as its stores do), 64-bit integers for
// integer programs (truncated to s32 where the program stores s32).
//
// Work split.  A CTA owns 4 adjacent outputs and all R rows, in chunks of 64
// rows.  Warps 1-7 (the workers) take 16-byte pieces of leaf rows (2 outputs
// of f64, 4 of a 4-byte type): for its (row, piece) positions of 8 chunks a
// worker copies the piece of every leaf into its own staging slots with
// cp.async, one commit group per position, so all of the group's copies are
// in flight together as in a plain streaming read.  It evaluates each
// position as soon as its own group has landed, with no barrier between
// workers.
//   f64 and f32 sums: the values go into the chunk's slot of a ring of value
//     buffers in shared memory, and warp 0 folds each output's values in
//     ascending row order as chunks become ready (one mbarrier per slot, one
//     arrival per worker warp).  The fold, one dependent add per row, runs
//     with 16 values prefetched into registers and frees each slot for the
//     chunk NS ahead.
//   integer sums: wrapping sums are associative, so each worker keeps partial
//     sums of its positions and the CTA combines them by shuffles, with no
//     chain at all.
//
// Other designs were measured first and lost to this one:
//   - a 2-D TMA tile (4 or 8 outputs x 64 rows), whose 32- and 64-byte box
//     rows came in at about one per 20 SM clocks;
//   - cp.async into shared raw tiles with a CTA-wide barrier per chunk, where
//     the per-chunk staging (stores, barrier, index arithmetic) took about
//     0.7 us per chunk and set the pace of the whole step;
//   - register staging, which needed more than 128 registers, so the spills
//     serialised the loads.
//
// Every wait is bounded; a wait that gives up records AMC_ERR_TIMEOUT in a
// device flag that the host reads after the step.
#include <atomic>
#include <cstring>
#include <type_traits>

#include "amc_internal.h"
#include "amc_tc.cuh"

namespace amc {

namespace {

__device__ int g_colfold_error;

struct ColForm {
  int32_t nops;            // 0: v = A; 1: v = A op1 B; 2: op2 applied as well
  int32_t op1, op2;        // 0 add, 1 subtract, 2 multiply
  int32_t rev2;            // v = C op2 t instead of t op2 C
  int32_t leaf[3];         // leaf read for A, B, C (0 for constants and unused operands)
  int32_t isk[3];          // the operand is a constant
  int32_t cvt1, cvt2;      // integer programs: truncate to s32 after op1 / op2
  double kf[3];            // float constants
  long long ki[3];         // integer constants
};

struct ColArgs {
  ColForm f;
  const void* leaf[2];
  long long pitch[2];      // elements between consecutive rows of each leaf
  long long O, R;
  int32_t nleaf, NS;
  int32_t op;              // AMC_RED_SUM or AMC_RED_MEAN
  void* out;
  int32_t out_dtype;
};

constexpr int kColOT = 4;             // outputs per CTA
constexpr int kColCH = 64;            // rows per chunk
constexpr int kColMaxNS = 16;         // ring slots at most
constexpr int kColWorkers = 224;      // warps 1-7
constexpr int kColG = 8;              // chunks whose loads a worker has in flight together
constexpr int kColVS = kColCH + 8;    // values per output in a slot: the 4 outputs land on two
                                      // bank halves, so a warp's stores take two wavefronts
constexpr int kColHead = 2 * kColMaxNS * 8;   // evaluated and freed barriers

__device__ __forceinline__ long long col_bini(int op, long long a, long long b) {
  const unsigned long long ua = (unsigned long long)a, ub = (unsigned long long)b;   // wrapping arithmetic
  const unsigned long long r = op == 2 ? ua * ub : op == 1 ? ua - ub : ua + ub;
  return (long long)r;
}

// The closed form on one element whose leaf values are x0 (leaf 0) and x1
// (leaf 1), returned as the bits the fold consumes: a double or a 64-bit integer.
template <typename LT>
__device__ __forceinline__ unsigned long long col_eval(const ColForm& F, LT x0, LT x1) {
  if (std::is_same<LT, int>::value) {
    const long long l0 = (long long)x0, l1 = (long long)x1;
    const long long a = F.isk[0] ? F.ki[0] : F.leaf[0] ? l1 : l0;
    const long long b = F.isk[1] ? F.ki[1] : F.leaf[1] ? l1 : l0;
    const long long c = F.isk[2] ? F.ki[2] : F.leaf[2] ? l1 : l0;
    long long t1 = col_bini(F.op1, a, b);
    if (F.cvt1) t1 = (long long)(int)t1;
    long long t2 = col_bini(F.op2, F.rev2 ? c : t1, F.rev2 ? t1 : c);
    if (F.cvt2) t2 = (long long)(int)t2;
    return (unsigned long long)(F.nops == 0 ? a : F.nops == 1 ? t1 : t2);
  } else {
    // the selectors are warp-uniform, so these branches never diverge and
    // each operation costs one instruction
    const double l0 = (double)x0, l1 = (double)x1;
    const double a = F.isk[0] ? F.kf[0] : F.leaf[0] ? l1 : l0;
    if (F.nops == 0) return (unsigned long long)__double_as_longlong(a);
    const double b = F.isk[1] ? F.kf[1] : F.leaf[1] ? l1 : l0;
    double t = F.op1 == 2 ? __dmul_rn(a, b) : F.op1 == 1 ? __dsub_rn(a, b) : __dadd_rn(a, b);
    if (std::is_same<LT, float>::value) t = (double)__double2float_rn(t);
    if (F.nops == 1) return (unsigned long long)__double_as_longlong(t);
    const double c = F.isk[2] ? F.kf[2] : F.leaf[2] ? l1 : l0;
    const double p = F.rev2 ? c : t, q = F.rev2 ? t : c;
    double u = F.op2 == 2 ? __dmul_rn(p, q) : F.op2 == 1 ? __dsub_rn(p, q) : __dadd_rn(p, q);
    if (std::is_same<LT, float>::value) u = (double)__double2float_rn(u);
    return (unsigned long long)__double_as_longlong(u);
  }
}

// Copy 16 bytes of leaf l at row r starting at output oc into dst (shared);
// bytes past the last output read as zero.
template <int ES>
__device__ __forceinline__ void col_copy(const ColArgs& a, int l, long long r, long long oc, void* dst) {
  const long long left = (a.O - oc) * ES;
  const int valid = left >= 16 ? 16 : left > 0 ? (int)left : 0;
  const char* src = (const char*)a.leaf[l];
  if (valid > 0) src += (r * a.pitch[l] + oc) * ES;   // nothing is read when valid == 0
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tc::smem_addr(dst)), "l"(src), "r"(valid)
               : "memory");
}
// Wait until at most n of this thread's newest commit groups are pending
// (n folds to a constant in the unrolled callers).
__device__ __forceinline__ void col_wait_group(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
  }
}

template <typename LT>
__device__ __forceinline__ LT col_elem(const uint4& v, int k) {
  if (sizeof(LT) == 8) {
    const unsigned long long b = k == 0 ? ((unsigned long long)v.y << 32 | v.x) : ((unsigned long long)v.w << 32 | v.z);
    LT r;
    memcpy(&r, &b, 8);
    return r;
  } else {
    const unsigned b = k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
    LT r;
    memcpy(&r, &b, 4);
    return r;
  }
}

// FOLD: 1 sum into f64; 2 f64 values summed into f32 (rounded after every
// step); 4 f32 values summed in f32; 3 integer sum.  LT: leaf element type.
template <typename LT, int FOLD>
__global__ void __launch_bounds__(256, 2) k_colfold(const __grid_constant__ ColArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int ES = sizeof(LT);
  constexpr int kPer = 16 / ES;                      // elements in one 16-byte piece
  constexpr int kPieces = kColOT / kPer;             // pieces per row (2 for f64, 1 for 4-byte types)
  constexpr int kGroupPieces = kColG * kColCH * kPieces;
  constexpr int kMaxPer = (kGroupPieces + kColWorkers - 1) / kColWorkers;
  const int NS = a.NS, nleaf = a.nleaf;
  uint64_t* evald = (uint64_t*)smem;
  uint64_t* freed = evald + kColMaxNS;
  unsigned long long* vals = (unsigned long long*)(smem + kColHead);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long o0 = (long long)blockIdx.x * kColOT;
  const long long R = a.R;
  const int nch = (int)((R + kColCH - 1) / kColCH);
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&evald[i], kColWorkers / 32);
      tc::mbar_init(&freed[i], 1);
    }
    tc::mbar_fence_init();
  }
  __syncthreads();
  if (FOLD == 3 && warp == 0) return;   // integer sums need no ordered chain (below)

  if (warp == 0) {
    // the fold: lane o (and its copies o + 4k, which keep the warp converged)
    // runs output o's chain over the chunks in row order
    const int o = lane % kColOT;
    double acc = 0.0;
    float accf = 0.f;
    unsigned long long acci = 0;
    bool ok = true;
    for (int j = 0; j < nch; ++j) {
      const int slot = j % NS;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&evald[slot], (j / NS) & 1))) {
        ok = false;
        break;
      }
      const int rc = (int)((R - (long long)j * kColCH) < kColCH ? (R - (long long)j * kColCH) : kColCH);
      const unsigned long long* vs = vals + (size_t)slot * kColOT * kColVS + o * kColVS;
      auto step = [&](unsigned long long bits) {
        const double x = __longlong_as_double((long long)bits);
        if (FOLD == 1) acc = __dadd_rn(acc, x);
        else if (FOLD == 2) acc = (double)__double2float_rn(__dadd_rn(acc, x));
        else if (FOLD == 4) accf = __fadd_rn(accf, (float)x);
        else acci += bits;
      };
      if (rc == kColCH) {
        // 16 values in registers while the next 16 load: the shared-memory
        // latency stays off the add chain
        const ulonglong2* v2 = (const ulonglong2*)vs;
        ulonglong2 cur[8], nxt[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) cur[k] = v2[k];
#pragma unroll
        for (int h = 0; h < kColCH / 16; ++h) {
          if (h + 1 < kColCH / 16) {
#pragma unroll
            for (int k = 0; k < 8; ++k) nxt[k] = v2[(h + 1) * 8 + k];
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            step(cur[k].x);
            step(cur[k].y);
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) cur[k] = nxt[k];
        }
      } else {
        for (int k = 0; k < rc; ++k) step(vs[k]);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&freed[slot]);
    }
    if (!ok) {
      if (lane == 0) atomicExch(&g_colfold_error, AMC_ERR_TIMEOUT);
      return;
    }
    if (lane < kColOT && o0 + lane < a.O) {
      const long long oi = o0 + lane;
      if (FOLD == 3) {
        if (a.out_dtype == AMC_S32) ((int*)a.out)[oi] = (int)(unsigned)acci;   // truncation commutes with +
        else ((long long*)a.out)[oi] = (long long)acci;
      } else {
        double r = FOLD == 4 ? (double)accf : acc;
        if (a.op == AMC_RED_MEAN) r = __ddiv_rn(r, (double)R);
        if (a.out_dtype == AMC_F32) ((float*)a.out)[oi] = __double2float_rn(r);
        else ((double*)a.out)[oi] = r;
      }
    }
    return;
  }

  // workers: position g of a group of kColG chunks is (chunk q, row, piece p)
  // with q = g / (64 * kPieces); consecutive lanes take consecutive pieces of
  // a row, then the next rows, so a warp's loads cover whole 32-byte sectors.
  // A worker copies the pieces of all leaves for its positions into its own
  // staging slots (cp.async, one commit group per position), then evaluates
  // each position as soon as its own group has landed: no barrier between
  // workers until the values are handed to the fold.
  const int wt = tid - 32;
  const ColForm& F = a.f;
  unsigned char* stage = smem + kColHead + (size_t)NS * kColOT * kColVS * 8;   // [kMaxPer][2][224] x 16 B
  auto stage_at = [&](int i, int l) { return stage + ((size_t)(i * 2 + l) * kColWorkers + wt) * 16; };
  if (FOLD == 3) {
    // wrapping integer sums are associative: each worker adds its own
    // positions' values, then the partial sums are combined (shuffles, then
    // one value per warp); the s32 result is the low half (truncation
    // commutes with +)
    unsigned long long part[kColOT] = {};
    for (int g0 = 0; g0 < nch; g0 += kColG) {
      const int gn = nch - g0 < kColG ? nch - g0 : kColG;
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        const int g = wt + i * kColWorkers;
        const int q = g / (kColCH * kPieces), rem = g % (kColCH * kPieces);
        const long long r = (long long)(g0 + q) * kColCH + rem / kPieces;
        const long long oc = o0 + (rem % kPieces) * kPer;
        if (q < gn && r < R) {
          for (int l = 0; l < nleaf; ++l) col_copy<ES>(a, l, r, oc, stage_at(i, l));
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      }
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        const int g = wt + i * kColWorkers;
        const int q = g / (kColCH * kPieces), rem = g % (kColCH * kPieces);
        const long long r = (long long)(g0 + q) * kColCH + rem / kPieces;
        col_wait_group(kMaxPer - 1 - i);
        if (q < gn && r < R) {
          const int ob = (rem % kPieces) * kPer;
          const uint4 v0 = *(const uint4*)stage_at(i, 0);
          const uint4 v1 = nleaf > 1 ? *(const uint4*)stage_at(i, 1) : v0;
#pragma unroll
          for (int k = 0; k < kPer; ++k)
            part[(ob + k) % kColOT] += col_eval<LT>(F, col_elem<LT>(v0, k), col_elem<LT>(v1, k));
        }
      }
    }
    unsigned long long* red = vals;   // [7 warps][4 outputs]
#pragma unroll
    for (int o = 0; o < kColOT; ++o) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part[o] += __shfl_xor_sync(0xffffffffu, part[o], off);
    }
    if (lane == 0) {
#pragma unroll
      for (int o = 0; o < kColOT; ++o) red[(warp - 1) * kColOT + o] = part[o];
    }
    tc::named_bar(1, kColWorkers);
    if (wt < kColOT && o0 + wt < a.O) {
      unsigned long long t = 0;
      for (int w = 0; w < kColWorkers / 32; ++w) t += red[w * kColOT + wt];
      if (a.out_dtype == AMC_S32) ((int*)a.out)[o0 + wt] = (int)(unsigned)t;
      else ((long long*)a.out)[o0 + wt] = (long long)t;
    }
    return;
  }
  bool ok = true;
  for (int g0 = 0; g0 < nch && ok; g0 += kColG) {
    const int gn = nch - g0 < kColG ? nch - g0 : kColG;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int g = wt + i * kColWorkers;
      const int q = g / (kColCH * kPieces), rem = g % (kColCH * kPieces);
      const long long r = (long long)(g0 + q) * kColCH + rem / kPieces;
      const long long oc = o0 + (rem % kPieces) * kPer;
      if (q < gn && r < R) {
        for (int l = 0; l < nleaf; ++l) col_copy<ES>(a, l, r, oc, stage_at(i, l));
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int q = 0; q < gn; ++q) {
      const int j = g0 + q, slot = j % NS;
      if (j >= NS && !tc::mbar_wait(&freed[slot], ((j / NS) - 1) & 1)) {   // the fold is done with chunk j - NS
        ok = false;
        break;
      }
      unsigned long long* vs = vals + (size_t)slot * kColOT * kColVS;
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        const int g = wt + i * kColWorkers;
        if (g / (kColCH * kPieces) == q) {
          col_wait_group(kMaxPer - 1 - i);   // this position's copies have landed
          const int rem = g % (kColCH * kPieces);
          const int row = rem / kPieces, ob = (rem % kPieces) * kPer;
          const uint4 v0 = *(const uint4*)stage_at(i, 0);
          const uint4 v1 = nleaf > 1 ? *(const uint4*)stage_at(i, 1) : v0;
#pragma unroll
          for (int k = 0; k < kPer; ++k)
            vs[(ob + k) * kColVS + row] = col_eval<LT>(F, col_elem<LT>(v0, k), col_elem<LT>(v1, k));
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&evald[slot]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");   // the staging slots are free for the next group
  }
  if (!ok) atomicExch(&g_colfold_error, AMC_ERR_TIMEOUT);
}

// ------------------------------------------------------------------ host side

// Closed form of the element program (see the file comment), or false.
// int_domain: an integer-only program over s32 leaves; round32: an f32
// program over f32 leaves, whose every operation is followed by its store
// to f32.  Otherwise a float program over f64 leaves, with no store at all.
bool col_form(const ReduceArgs& a, bool int_domain, bool round32, ColForm& F) {
  memset(&F, 0, sizeof F);
  struct Sym {
    int kind;   // 0 leaf, 1 constant, 2 result of op1, 3 result of op2
    int leaf;
    double kf;
    long long ki;
  };
  Sym st[4];
  int sp = 0, nops = 0;
  bool rnd1 = false, rnd2 = false;
  auto set_operand = [&](int slot, const Sym& x) {
    F.isk[slot] = x.kind == 1;
    F.leaf[slot] = x.kind == 0 ? x.leaf : 0;
    F.kf[slot] = x.kf;
    F.ki[slot] = x.ki;
  };
  for (int pc = 0; pc < a.prog.n; ++pc) {
    const amc_insn& I = a.prog.code[pc];
    switch (I.op) {
      case AMC_OP_LOAD:
        if (sp >= 4 || I.a < 0 || I.a >= a.nleaf) return false;
        st[sp++] = Sym{0, I.a, 0.0, 0};
        break;
      case AMC_OP_CONST:
        if (sp >= 4 || int_domain) return false;
        st[sp++] = Sym{1, 0, I.imm, 0};
        break;
      case AMC_OP_ICONST:
        // in a float program an exact constant meets a float leaf, which
        // makes the result inexact: it acts as its double value
        if (sp >= 4) return false;
        st[sp++] = Sym{1, 0, (double)(long long)I.imm, (long long)I.imm};
        break;
      case AMC_OP_CVT: {
        if (sp < 1) return false;
        const Sym& t = st[sp - 1];
        if (t.kind >= 2) {
          if (int_domain) {
            if (I.a == AMC_S32) (t.kind == 2 ? F.cvt1 : F.cvt2) = 1;
            else if (I.a != AMC_S64) return false;
          } else if (I.a == AMC_F32) {
            if (!round32) return false;
            (t.kind == 2 ? rnd1 : rnd2) = true;
          } else if (I.a != AMC_F64) {   // a store to f64 leaves a double as it is
            return false;
          }
        } else if (t.kind == 0) {
          // a store of a leaf value to its own type (or a wider one) changes nothing
          const bool same = int_domain ? (I.a == AMC_S32 || I.a == AMC_S64)
                                       : (I.a == AMC_F64 || (round32 && I.a == AMC_F32));
          if (!same) return false;
        } else if (!(!int_domain && I.a == AMC_F64)) {
          return false;
        }
        break;
      }
      case AMC_OP_ADD:
      case AMC_OP_SUB:
      case AMC_OP_MUL: {
        if (sp < 2) return false;
        const int opk = I.op == AMC_OP_ADD ? 0 : I.op == AMC_OP_SUB ? 1 : 2;
        const Sym y = st[--sp], x = st[--sp];
        if (nops == 0 && x.kind <= 1 && y.kind <= 1 && !(x.kind == 1 && y.kind == 1)) {
          F.op1 = opk;
          set_operand(0, x);
          set_operand(1, y);
          st[sp++] = Sym{2, 0, 0.0, 0};
          nops = 1;
        } else if (nops == 1 && (x.kind == 2) != (y.kind == 2) && (x.kind <= 2 && y.kind <= 2)) {
          F.op2 = opk;
          F.rev2 = y.kind == 2;
          set_operand(2, y.kind == 2 ? x : y);
          st[sp++] = Sym{3, 0, 0.0, 0};
          nops = 2;
        } else {
          return false;
        }
        break;
      }
      default:
        return false;
    }
  }
  if (sp != 1) return false;
  if (nops == 0) {
    if (st[0].kind != 0) return false;
    set_operand(0, st[0]);
  }
  if (st[0].kind != (nops == 0 ? 0 : nops + 1)) return false;
  if (round32 && ((nops >= 1 && !rnd1) || (nops == 2 && !rnd2))) return false;
  // unused operands read leaf 0 (a valid tile) and are never selected
  if (nops < 2) { F.leaf[2] = 0; F.isk[2] = 0; }
  if (nops < 1) { F.leaf[1] = 0; F.isk[1] = 0; }
  F.nops = nops;
  return true;
}

std::atomic<long long> g_colfold_launches{0};

template <typename LT, int FOLD>
int colfold_go(const ColArgs& ca, size_t smem, cudaStream_t s) {
  static bool attr_set = false;
  if (!attr_set) {
    AMC_CUDA(cudaFuncSetAttribute(k_colfold<LT, FOLD>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
    attr_set = true;
  }
  const unsigned grid = (unsigned)((ca.O + kColOT - 1) / kColOT);
  k_colfold<LT, FOLD><<<grid, 256, smem, s>>>(ca);
  AMC_CUDA(cudaGetLastError());
  g_colfold_launches.fetch_add(1, std::memory_order_relaxed);
  return AMC_OK;
}

}  // namespace

// Launch the column fold for `a`, or return AMC_ERR_UNSUPPORTED (nothing
// launched, no error recorded) when the reduction is not of its kind.
int launch_colfold(const ReduceArgs& a, cudaStream_t s) {
  if (a.orank != 1 || a.rrank != 1 || a.nleaf < 1 || a.nleaf > 2 || a.O < 1 || a.R < 1) return AMC_ERR_UNSUPPORTED;
  if (a.R >= (1ll << 31) || a.O >= (1ll << 31)) return AMC_ERR_UNSUPPORTED;
  const int D = a.leaf_o[0].dtype;
  if (D != AMC_F64 && D != AMC_F32 && D != AMC_S32) return AMC_ERR_UNSUPPORTED;
  const int esize = D == AMC_F64 ? 8 : 4;
  // 16-byte copies: every row of 4 outputs starts on a 16-byte boundary
  for (int l = 0; l < a.nleaf; ++l)
    if (a.leaf_o[l].dtype != D || a.leaf_o[l].strides[0] != 1 || a.leaf_r[l][0] <= 0 ||
        ((uintptr_t)a.leaf_o[l].ptr & 15) || ((a.leaf_r[l][0] * esize) & 15))
      return AMC_ERR_UNSUPPORTED;
  const bool sumlike = a.op == AMC_RED_SUM || a.op == AMC_RED_MEAN;
  if (!sumlike) return AMC_ERR_UNSUPPORTED;
  int fold = 0;
  bool int_domain = false, round32 = false;
  if (D == AMC_S32) {
    if (a.prog.all_float || a.op != AMC_RED_SUM) return AMC_ERR_UNSUPPORTED;
    if ((a.src_dtype != AMC_S32 && a.src_dtype != AMC_S64) || (a.out_dtype != AMC_S32 && a.out_dtype != AMC_S64))
      return AMC_ERR_UNSUPPORTED;
    for (int pc = 0; pc < a.prog.n; ++pc)
      if (a.prog.code[pc].op == AMC_OP_CONST) return AMC_ERR_UNSUPPORTED;
    int_domain = true;
    fold = 3;
  } else {
    // float leaves: every value is inexact; integer constants are allowed
    // (they meet a leaf), stores to integer types are not (col_form)
    if (a.src_dtype != D) return AMC_ERR_UNSUPPORTED;
    round32 = D == AMC_F32;
    if (a.out_dtype == AMC_F64) fold = 1;
    else if (a.out_dtype == AMC_F32) fold = D == AMC_F32 ? 4 : 2;
    else return AMC_ERR_UNSUPPORTED;
  }
  ColArgs ca;
  memset(&ca, 0, sizeof ca);
  if (!col_form(a, int_domain, round32, ca.f)) return AMC_ERR_UNSUPPORTED;
  const int nch = (int)((a.R + kColCH - 1) / kColCH);
  ca.NS = nch < kColMaxNS ? nch : kColMaxNS;
  ca.nleaf = a.nleaf;
  for (int l = 0; l < a.nleaf; ++l) {
    ca.leaf[l] = a.leaf_o[l].ptr;
    ca.pitch[l] = a.leaf_r[l][0];
  }
  ca.O = a.O;
  ca.R = a.R;
  ca.op = a.op;
  ca.out = a.out;
  ca.out_dtype = a.out_dtype;
  // value ring, then each worker's staging slots: 16 bytes per leaf for each
  // of its positions in a group of chunks
  const int pieces = esize == 8 ? 2 : 1;
  const int max_per = (kColG * kColCH * pieces + kColWorkers - 1) / kColWorkers;
  const size_t smem = kColHead + (size_t)ca.NS * kColOT * kColVS * 8 + (size_t)max_per * 2 * kColWorkers * 16;
  switch (fold) {
    case 1: return D == AMC_F64 ? colfold_go<double, 1>(ca, smem, s) : colfold_go<float, 1>(ca, smem, s);
    case 2: return colfold_go<double, 2>(ca, smem, s);
    case 4: return colfold_go<float, 4>(ca, smem, s);
    default: return colfold_go<int, 3>(ca, smem, s);
  }
}

long long colfold_launch_count() { return g_colfold_launches.load(std::memory_order_relaxed); }

int colfold_check_error() {
  int e = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&e, g_colfold_error, sizeof(int)));
  if (e) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_colfold_error, &z, sizeof(int)));
    return fail(e, "column fold: a bounded wait for a chunk gave up");
  }
  return AMC_OK;
}

}  // namespace amc

extern "C" int amc_colfold_launch_count(int64_t* count) {
  if (!count) return amc::fail(AMC_ERR_INVALID, "amc_colfold_launch_count: null count");
  *count = amc::colfold_launch_count();
  return AMC_OK;
}
