// C-ABI entry points: plan a convolution, lay out the workspace, and run the passes.
//
// cnd_forward replaces torch_convnd::conv_nd's CUDA kernel (reference
// src/torch_convnd/csrc/convnd.cpp:305-343): pack x to channels-last, pack W, one
// tcgen05 implicit-GEMM launch whose epilogue adds the bias and writes channels-first y.
// cnd_backward replaces conv_nd_backward (convnd.cpp:345-415, convnd_mixed.cpp:11-59):
// one pack of dy (which also yields the bias-gradient partials), dgrad as a forward
// pass over dy with flipped/transposed weights (stride 1), and wgrad as a split-K
// tcgen05 pass followed by an ordered reduction. Anything outside the tensor-core path
// runs on the generic CUDA-core kernels. There is no CPU path.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "generic.cuh"
#include "internal.h"
#include "pack.cuh"
#include "fprop.cuh"
#include "tc_conv.cuh"

namespace cnd {

__device__ unsigned int g_error_word;

// Workspace of cnd_forward_noalloc: a fixed device array instead of an allocation.
static __device__ __align__(256) unsigned char g_forward_scratch[CND_NOALLOC_SCRATCH_BYTES];

namespace {

std::atomic<int64_t> g_launches{0};

uint64_t wait_timeout_ns() {
  static uint64_t value = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    uint64_t ms = 2000;
    if (const char* env = std::getenv("CND_WAIT_TIMEOUT_MS")) {
      const long long parsed = std::atoll(env);
      if (parsed > 0) ms = static_cast<uint64_t>(parsed);
    }
    value = ms * 1000000ull;
  });
  return value;
}

}  // namespace

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

unsigned int* device_error_word() {
  static std::mutex mutex;
  static unsigned int* words[128] = {};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 128) return nullptr;
  std::lock_guard<std::mutex> lock(mutex);
  if (words[device] == nullptr) {
    void* address = nullptr;
    if (cudaGetSymbolAddress(&address, g_error_word) == cudaSuccess) {
      words[device] = static_cast<unsigned int*>(address);
    }
  }
  return words[device];
}

namespace {

// ---- optional per-pass CUDA-event timing (benchmark support) ----
std::mutex g_timing_mutex;
bool g_timing = false;
struct TimingRecord {
  int kind;
  cudaEvent_t start, stop;
};
std::vector<TimingRecord> g_timings;

// Brackets one pass with events on its stream when timing is enabled.
class TimedPass {
 public:
  TimedPass(int kind, cudaStream_t stream) : stream_(stream) {
    std::lock_guard<std::mutex> lock(g_timing_mutex);
    if (!g_timing) return;
    record_.kind = kind;
    if (cudaEventCreate(&record_.start) != cudaSuccess) return;
    if (cudaEventCreate(&record_.stop) != cudaSuccess) {
      cudaEventDestroy(record_.start);
      return;
    }
    active_ = true;
    cudaEventRecord(record_.start, stream_);
  }
  ~TimedPass() {
    if (!active_) return;
    cudaEventRecord(record_.stop, stream_);
    std::lock_guard<std::mutex> lock(g_timing_mutex);
    g_timings.push_back(record_);
  }

 private:
  cudaStream_t stream_;
  TimingRecord record_{};
  bool active_ = false;
};

constexpr size_t kAlign = 1024;

size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

int operand_type(int dtype) {
  if (dtype == CND_BF16) return kOpBF16;
  if (dtype == CND_F16) return kOpF16;
  return kOpF32;
}

int element_bytes(int dtype) {
  if (dtype == CND_F64) return 8;
  if (dtype == CND_F32) return 4;
  return 2;
}

// Channel count of a packed channels-last operand: rows of 32, 64 or 128 bytes (one
// swizzle atom), or a multiple of 128 bytes.
int64_t pad_channels(int op, int64_t c, int64_t minimum) {
  if (c < minimum) c = minimum;
  const int64_t unit = op == kOpF32 ? 8 : 16;  // 32 bytes
  if (c <= unit) return unit;
  if (c <= 2 * unit) return 2 * unit;
  if (c <= 4 * unit) return 4 * unit;
  return (c + 4 * unit - 1) / (4 * unit) * (4 * unit);
}

int64_t round16(int64_t v) { return (v + 15) / 16 * 16; }

struct Region {
  size_t offset = 0, bytes = 0;
};

struct Plan {
  bool tensor_cores = false;  // dtype allows the tcgen05 path at all
  int op = 0;
  int split3 = 0;
  int pack_mode = 0;
  int parts = 1;
  // Channel groups of the tensor-core passes. Grouped problems whose per-group channels
  // are thin run as one dense problem with block-diagonal weights (bd = the problem's
  // group count): the packed rows then hold every channel once instead of each group
  // padded to a 32-byte row, and the MMAs see all channels at once. cin_g / cout_g are
  // the channels per pass group (all channels when bd > 1).
  int64_t groups = 1;
  int bd = 1;
  int64_t cin_g = 0, cout_g = 0;
  int64_t x_pad = 0, dy_pad = 0;
  // Channels-last activations (cnd_problem.layout) whose rows already are the packed
  // operand rows (16-bit, one pass group, channel count equal to the padded width) are
  // read in place: no layout pass and no workspace copy.
  bool x_cl = false, y_cl = false, x_direct = false, dy_direct = false;
  // Fused activation (cnd_problem.layout bits 8-15): the forward epilogue applies it, the
  // backward's dy pack multiplies by its derivative (so dy is always packed); dz_raw holds
  // dy * act'(pre) in dy's layout when a generic pass needs the unpacked product.
  int act = 0;
  Region dz_raw;
  bool fast_fwd = false, fast_dgrad = false, fast_wgrad = false;
  // float32 dgrad on bfloat16 hi + lo operand parts (three kind::f16 products) instead
  // of 3xTF32, when that halves the K steps (dy channels a multiple of 16). Its packed dy
  // is the weight gradient's (wg_dy).
  bool dgrad_bf16 = false;
  ConvPass fwd{}, dgrad{};
  FpropPlan fwd_plan{}, dgrad_plan{};
  // Strided dgrad as phase sub-convolutions (one per residue class of dx positions modulo
  // the strides): nphase > 0 replaces the single dgrad pass; phase_empty: some residue
  // class has no tap, so dx is zeroed before the phases write theirs.
  static constexpr int kMaxPhases = 16;
  int nphase = 0;
  bool phase_empty = false;
  ConvPass phase[kMaxPhases]{};
  FpropPlan phase_plan[kMaxPhases]{};
  PackWeightArgs phase_taps[kMaxPhases]{};
  Region w_phase[kMaxPhases], w_phase_small[kMaxPhases];
  WgradPass wgrad{};
  // weight-gradient operands: 16-bit problems reuse the packed x / dy; float32 problems pack
  // x and dy again as 3 (3xtf32 mode) or 2 (tf32 mode) bfloat16 terms.
  int wg_op = 0, wg_parts = 1, wg_mode = 0;
  int64_t wg_x_pad = 0, wg_dy_pad = 0;
  // wg_fold > 1: the weight gradient reads x with the last axis's wg_fold taps folded
  // into its channels (k1 taps per channel group instead of whole padded rows fill the
  // M tiles of thin-channel layers); the pass sees that axis as a one-tap axis of
  // wg_fold_last_dst positions, and wg_x holds wg_x_spatial positions per image.
  int wg_fold = 1;
  int64_t wg_fold_last_src = 0, wg_fold_last_dst = 0, wg_fold_d = 1, wg_fold_p = 0;
  int64_t wg_x_spatial = 0;
  // workspace
  Region x_pack, x_pack_small, w_fwd, w_fwd_small, dy_pack, dy_pack_small, w_dg, w_dg_small,
      partial, bias_partial, bias_chunks;
  Region wg_x[3], wg_dy[3];
  size_t total = 0;
};

// Spatial geometry of the tensor-core passes after axis reduction.
struct Axes {
  int rank = 0;
  int64_t in[CND_MAX_RANK], out[CND_MAX_RANK], k[CND_MAX_RANK], s[CND_MAX_RANK],
      d[CND_MAX_RANK], p[CND_MAX_RANK];
  void push(int64_t in_, int64_t out_, int64_t k_, int64_t s_, int64_t d_, int64_t p_) {
    in[rank] = in_;
    out[rank] = out_;
    k[rank] = k_;
    s[rank] = s_;
    d[rank] = d_;
    p[rank] = p_;
    ++rank;
  }
};

// The reference's without_unit_axes (src/torch_convnd/csrc/convnd.h:32-48): an axis with
// one sample, a one-tap kernel and no padding puts every element at coordinate 0, so it
// is dropped from the index arithmetic (one axis is always kept). Memory layouts and
// volumes are unchanged: the packed operands and the outputs do not depend on it.
Axes without_unit_axes(const cnd_problem& p) {
  Axes a;
  for (int axis = 0; axis < p.rank; ++axis) {
    const bool unit = p.input[axis] == 1 && p.kernel[axis] == 1 && p.padding[axis] == 0;
    if (unit && (a.rank > 0 || axis + 1 < p.rank)) continue;
    a.push(p.input[axis], p.output[axis], p.kernel[axis], p.stride[axis], p.dilation[axis],
           p.padding[axis]);
  }
  return a;
}

// Adjacent pointwise axes (kernel 1, stride 1, padding 0: the output coordinate equals the
// input coordinate and every tap sits at offset 0) address memory exactly like one axis of
// their product extent, so each run of them becomes one axis. The planners see a longer
// innermost extent (c5's k = (3,3,1,1) layer: [16,16,64] instead of [16,16,8,8]).
Axes merge_pointwise(const Axes& a) {
  Axes m;
  bool last_pointwise = false;
  for (int axis = 0; axis < a.rank; ++axis) {
    const bool pointwise = a.k[axis] == 1 && a.s[axis] == 1 && a.p[axis] == 0;
    if (pointwise && last_pointwise) {
      m.in[m.rank - 1] *= a.in[axis];
      m.out[m.rank - 1] *= a.out[axis];
      continue;
    }
    m.push(a.in[axis], a.out[axis], a.k[axis], a.s[axis], pointwise ? 1 : a.d[axis],
           a.p[axis]);
    last_pointwise = pointwise;
  }
  return m;
}

void fill_spatial(const Axes& ax, int64_t* in, int64_t* out, int64_t* k, int64_t* s,
                  int64_t* d, int64_t* pad) {
  for (int a = 0; a < ax.rank; ++a) {
    in[a] = ax.in[a];
    out[a] = ax.out[a];
    k[a] = ax.k[a];
    s[a] = ax.s[a];
    d[a] = ax.d[a];
    pad[a] = ax.p[a];
  }
}

// Plans a forward-type pass over each axis variant that fits the kernels and keeps the
// one the cost model scores best.
bool plan_best(ConvPass* pass, FpropPlan* plan, const Axes* const* variants, int count,
               bool dgrad) {
  bool found = false;
  double best = 0.0;
  for (int v = 0; v < count; ++v) {
    const Axes& ax = *variants[v];
    if (ax.rank > kMaxFastRank) continue;
    ConvPass trial = *pass;
    trial.rank = ax.rank;
    for (int a = 0; a < ax.rank; ++a) {
      trial.in[a] = dgrad ? ax.out[a] : ax.in[a];
      trial.out[a] = dgrad ? ax.in[a] : ax.out[a];
      trial.k[a] = ax.k[a];
      trial.s[a] = dgrad ? 1 : ax.s[a];
      trial.d[a] = ax.d[a];
      trial.p[a] = dgrad ? ax.d[a] * (ax.k[a] - 1) - ax.p[a] : ax.p[a];
    }
    FpropPlan candidate;
    if (!plan_fprop(trial, &candidate)) continue;
    if (!found || candidate.score < best) {
      found = true;
      best = candidate.score;
      *pass = trial;
      *plan = candidate;
    }
  }
  return found;
}

Region take(size_t* cursor, size_t bytes) {
  Region r;
  r.offset = *cursor;
  r.bytes = bytes;
  *cursor = align_up(*cursor + bytes);
  return r;
}

int gcd_int(int64_t a, int64_t b) {
  while (b != 0) {
    const int64_t t = a % b;
    a = b;
    b = t;
  }
  return static_cast<int>(a);
}

// Splits the input gradient of a strided problem into phase sub-convolutions. Residue
// class r (per axis, 0 <= r < s) holds dx positions s * j + r; the taps that reach it are
// those with (r + p - t * d) divisible by s, an arithmetic progression of step s / gcd(d, s)
// whose dy offsets (r + p - t * d) / s step by d / gcd(d, s). In dy coordinates the class is
// a stride-1 convolution with that many taps, dilation d / g and padding -(smallest offset),
// taps ordered by ascending offset (descending t), written to the strided sub-grid
// (the reference's fold, convnd_cuda.cu:147-169 / input_column_offset convnd.h:79-104,
// as dense sub-convolutions). False when there are too many classes or a class does not
// fit the tcgen05 pass.
bool plan_phases(const Axes& ax, const ConvPass& templ, Plan* plan) {
  int64_t classes = 1;
  for (int a = 0; a < ax.rank; ++a) classes *= ax.s[a];
  if (classes > Plan::kMaxPhases || ax.rank > kMaxFastRank) return false;
  plan->nphase = 0;
  plan->phase_empty = false;
  for (int64_t c = 0; c < classes; ++c) {
    int64_t rest = c;
    ConvPass ph = templ;
    PackWeightArgs taps{};
    ph.rank = ax.rank;
    ph.out_strided = 1;
    taps.phase_rank = ax.rank;
    bool empty = false;
    for (int a = ax.rank - 1; a >= 0; --a) {
      const int64_t s = ax.s[a], r = rest % s;
      rest /= s;
      int64_t count = 0, t_last = -1;
      for (int64_t t = 0; t < ax.k[a]; ++t) {
        if ((r + ax.p[a] - t * ax.d[a]) % s == 0) {
          ++count;
          t_last = t;
        }
      }
      const int64_t g = gcd_int(ax.d[a], s);
      ph.in[a] = ax.out[a];
      ph.out[a] = (ax.in[a] - r + s - 1) / s;
      ph.k[a] = count > 0 ? count : 1;
      ph.s[a] = 1;
      ph.d[a] = ax.d[a] / g;
      ph.p[a] = count > 0 ? -((r + ax.p[a] - t_last * ax.d[a]) / s) : 0;
      ph.out_mul[a] = s;
      ph.out_add[a] = r;
      ph.out_full[a] = ax.in[a];
      taps.k_sub[a] = static_cast<int>(ph.k[a]);
      taps.k_full[a] = static_cast<int>(ax.k[a]);
      taps.tap_first[a] = static_cast<int>(t_last);
      taps.tap_step[a] = -static_cast<int>(s / g);
      if (count == 0 || ph.out[a] <= 0) empty = true;
    }
    if (empty) {
      plan->phase_empty = true;
      continue;
    }
    const int i = plan->nphase;
    if (!plan_fprop(ph, &plan->phase_plan[i])) return false;
    plan->phase[i] = ph;
    plan->phase_taps[i] = taps;
    ++plan->nphase;
  }
  return plan->nphase > 0;
}

// Decides the kernel family of every pass and the workspace layout.
// `forward` selects the forward plan; otherwise `mask` selects the backward passes.
void make_plan(const cnd_problem& p, bool forward, const int32_t* mask, Plan* plan) {
  *plan = Plan();
  const Axes reduced = without_unit_axes(p);
  const Axes merged = merge_pointwise(reduced);
  const Axes* variants[2] = {&reduced, &merged};
  const int nvariants = merged.rank < reduced.rank ? 2 : 1;
  plan->groups = p.groups;
  plan->cin_g = p.channels / p.groups;
  plan->cout_g = p.output_channels / p.groups;
  const bool low = p.dtype == CND_BF16 || p.dtype == CND_F16;
  const bool f32_tensor = p.dtype == CND_F32 && p.fp32_mode != CND_FP32_SIMT;
  plan->tensor_cores = (low || f32_tensor) && merged.rank <= kMaxFastRank && p.batch > 0;
  if (!plan->tensor_cores) {
    // generic kernels only: the activation backward needs its product materialised
    plan->act = (p.layout >> CND_LAYOUT_ACT_SHIFT) & 0xff;
    if (!forward && plan->act != 0 && p.batch > 0) {
      size_t cursor = 0;
      plan->dz_raw = take(&cursor, static_cast<size_t>(p.batch * p.output_channels *
                                                       p.output_volume) *
                                       element_bytes(p.dtype));
      plan->total = cursor;
    }
    return;
  }
  plan->op = operand_type(p.dtype);
  plan->split3 = (p.dtype == CND_F32 && p.fp32_mode == CND_FP32_3XTF32) ? 1 : 0;
  plan->pack_mode = p.dtype == CND_F32 ? (plan->split3 ? 1 : 2) : 0;
  plan->parts = plan->split3 ? 2 : 1;
  const size_t es = element_bytes(p.dtype);
  if (p.groups > 1 && p.channels <= 64 && p.output_channels <= 64) {
    // Dense when padding each group to its own row costs more bytes than one row of all
    // channels (the extra block-diagonal products are cheaper than thin MMAs).
    const bool thin =
        p.groups * pad_channels(plan->op, plan->cin_g, 1) >
            pad_channels(plan->op, p.channels, 1) ||
        p.groups * pad_channels(plan->op, plan->cout_g, 16) >
            pad_channels(plan->op, p.output_channels, 16);
    if (thin) {
      plan->bd = static_cast<int>(p.groups);
      plan->groups = 1;
      plan->cin_g = p.channels;
      plan->cout_g = p.output_channels;
    }
  }
  plan->x_pad = pad_channels(plan->op, plan->cin_g, 1);
  plan->dy_pad = pad_channels(plan->op, plan->cout_g, 16);
  plan->x_cl = (p.layout & CND_LAYOUT_X_CL) != 0;
  plan->y_cl = (p.layout & CND_LAYOUT_Y_CL) != 0;
  plan->x_direct = plan->x_cl && low && plan->groups == 1 && p.channels == plan->x_pad;
  plan->act = (p.layout >> CND_LAYOUT_ACT_SHIFT) & 0xff;
  plan->dy_direct = plan->act == 0 && plan->y_cl && low && plan->groups == 1 &&
                    p.output_channels == plan->dy_pad;
  const int64_t taps = p.kernel_volume;
  size_t cursor = 0;

  if (forward) {
    ConvPass& f = plan->fwd;
    f.batch = p.batch;
    f.groups = plan->groups;
    f.c_pad = static_cast<int>(plan->x_pad);
    f.n_real = static_cast<int>(plan->cout_g);
    f.n_pad = static_cast<int>(round16(plan->cout_g));
    f.op = plan->op;
    f.split3 = plan->split3;
    f.out_dtype = p.dtype;
    f.out_cl = plan->y_cl ? 1 : 0;
    f.activation = plan->act;  // the planner reserves staging for the pre-activation
    plan->fast_fwd =
        plan->cout_g <= 256 && plan_best(&f, &plan->fwd_plan, variants, nvariants, false);
    if (plan->fast_fwd) {
      const size_t act =
          static_cast<size_t>(p.batch * plan->groups * p.input_volume) * f.c_pad * es;
      const size_t wts = static_cast<size_t>(plan->groups * taps * f.n_pad * f.c_pad) * es;
      if (!plan->x_direct) plan->x_pack = take(&cursor, act);
      if (plan->split3) plan->x_pack_small = take(&cursor, act);
      plan->w_fwd = take(&cursor, wts);
      if (plan->split3) plan->w_fwd_small = take(&cursor, wts);
    }
    plan->total = cursor;
    return;
  }

  // ---- backward ----
  bool strided = false, wide_pad = false;
  for (int a = 0; a < p.rank; ++a) {
    if (p.stride[a] != 1) strided = true;
    if (p.padding[a] > p.dilation[a] * (p.kernel[a] - 1)) wide_pad = true;
  }
  if (mask[0]) {
    ConvPass& dg = plan->dgrad;
    dg.batch = p.batch;
    dg.groups = plan->groups;
    dg.c_pad = static_cast<int>(plan->dy_pad);
    dg.n_real = static_cast<int>(plan->cin_g);
    dg.n_pad = static_cast<int>(round16(plan->cin_g));
    dg.op = plan->op;
    dg.split3 = plan->split3;
    dg.out_dtype = p.dtype;
    dg.out_cl = plan->x_cl ? 1 : 0;
    const bool dgrad_ok = !strided && !wide_pad && plan->cin_g <= 256;
    if (strided && plan->cin_g <= 256) {
      // Strided: phase sub-convolutions over the packed dy (float32 problems on the
      // bf16 hi/lo parts when that halves the K steps, as below).
      ConvPass templ = dg;
      const int64_t bf16_pad = pad_channels(kOpBF16, plan->cout_g, 16);
      if (plan->split3 && bf16_pad / 16 < plan->dy_pad / 8) {
        // split3 stays set: two operand parts, three products (the 2xBF16 kernel)
        templ.op = kOpBF16;
        templ.c_pad = static_cast<int>(bf16_pad);
        plan->dgrad_bf16 = true;
      }
      if (plan_phases(reduced, templ, plan)) {
        dg = templ;
        plan->fast_dgrad = true;
      } else {
        plan->dgrad_bf16 = false;
        plan->nphase = 0;
      }
    }
    // One bf16 K step covers 16 dy channels, one TF32 step 8: the bf16 parts win when
    // they need fewer K steps (dy channels >= 16); below that they would only lose
    // precision.
    const int64_t bf16_pad = pad_channels(kOpBF16, plan->cout_g, 16);
    if (dgrad_ok && plan->split3 && bf16_pad / 16 < plan->dy_pad / 8) {
      ConvPass bf = dg;
      bf.op = kOpBF16;
      bf.c_pad = static_cast<int>(bf16_pad);
      if (plan_best(&bf, &plan->dgrad_plan, variants, nvariants, true)) {
        dg = bf;
        plan->dgrad_bf16 = true;
        plan->fast_dgrad = true;
      }
    }
    if (!plan->dgrad_bf16 && plan->nphase == 0) {
      plan->fast_dgrad = dgrad_ok && plan_best(&dg, &plan->dgrad_plan, variants, nvariants, true);
    }
  }
  const bool f32 = p.dtype == CND_F32;
  plan->wg_op = f32 ? kOpBF16 : plan->op;
  // float32 weight gradients run as bf16 hi + lo parts (three cross products, ~16
  // significant bits per operand): at c4's full size their dW rel-L2 error is 1.3e-5,
  // against 2.5e-5 with three parts and six products, which cost twice the MMAs.
  plan->wg_parts = f32 ? 2 : 1;
  plan->wg_mode = f32 ? 4 : 0;
  plan->wg_x_pad = f32 ? pad_channels(kOpBF16, plan->cin_g, 1) : plan->x_pad;
  plan->wg_dy_pad = f32 ? pad_channels(kOpBF16, plan->cout_g, 16) : plan->dy_pad;
  plan->wg_x_spatial = p.input_volume;
  if (mask[1] && plan->bd == 1 && reduced.rank >= 1) {
    // Fold the last axis's taps into the channels when that fills the weight-gradient
    // M tiles markedly better. The kernel's M tile is 128 rows of tap atoms, one padded
    // channel row each; halo plans take the a1 taps as atoms (k1 of every ceil(k1 / atoms)
    // * atoms used), the others consecutive taps. c4 (8 channels as 16-wide bf16 parts,
    // k1 = 3): 3/8 * 8/16 of the rows used, folded (24 channels in 32) 3/4 * 24/32.
    const int L = reduced.rank - 1;
    const int64_t k_last = reduced.k[L];
    const int64_t c_fold = k_last * plan->cin_g;
    const int fold_op = f32 ? kOpBF16 : plan->op;
    const bool whole_chunks = plan->cin_g == 8 || plan->cin_g == 16 || plan->cin_g == 32;
    if (k_last >= 2 && c_fold <= 64 && whole_chunks && reduced.out[L] >= 1) {
      const int64_t k1 = reduced.rank >= 2 ? reduced.k[L - 1] : 1;
      const bool halo = reduced.rank >= 2 && k1 >= 2 && reduced.s[L - 1] == 1;
      auto m_use = [&](int64_t c_real, int64_t c_pad, int64_t taps_now) {
        const int64_t atoms = 128 / c_pad;
        double used;
        if (halo) {
          used = double(k1) / double((k1 + atoms - 1) / atoms * atoms);
        } else {
          used = double(taps_now) / double((taps_now + atoms - 1) / atoms * atoms);
        }
        return used * double(c_real) / double(c_pad);
      };
      const int64_t pad_fold = pad_channels(fold_op, c_fold, 1);
      if (m_use(c_fold, pad_fold, taps / k_last) >
          1.25 * m_use(plan->cin_g, plan->wg_x_pad, taps)) {
        plan->wg_fold = static_cast<int>(k_last);
        plan->wg_x_pad = pad_fold;
        plan->wg_fold_last_src = reduced.in[L];
        plan->wg_fold_last_dst = (reduced.out[L] - 1) * reduced.s[L] + 1;
        plan->wg_fold_d = reduced.d[L];
        plan->wg_fold_p = reduced.p[L];
        plan->wg_x_spatial = p.input_volume / reduced.in[L] * plan->wg_fold_last_dst;
      }
    }
  }
  if (mask[1]) {
    WgradPass& wg = plan->wgrad;
    wg.rank = reduced.rank;
    wg.batch = p.batch;
    wg.groups = plan->groups;
    fill_spatial(reduced, wg.in, wg.out, wg.k, wg.s, wg.d, wg.p);
    if (plan->wg_fold > 1) {
      // the folded axis: one tap at offset 0 over the shifted copies' positions
      const int L = reduced.rank - 1;
      wg.in[L] = plan->wg_fold_last_dst;
      wg.k[L] = 1;
      wg.d[L] = 1;
      wg.p[L] = 0;
    }
    wg.c_pad = static_cast<int>(plan->wg_x_pad);
    wg.cin_real = static_cast<int>(plan->cin_g * plan->wg_fold);
    wg.n_pad = static_cast<int>(plan->wg_dy_pad);
    wg.n_real = static_cast<int>(plan->cout_g);
    wg.op = plan->wg_op;
    wg.parts = plan->wg_parts;
    plan->fast_wgrad = plan->cout_g <= 256 && wgrad_pass_supported(wg);
    if (plan->fast_wgrad) wg.splits = plan_wgrad_splits(wg, 0);
    if (wg.splits <= 0) plan->fast_wgrad = false;
  }
  const bool need_dy = (plan->fast_dgrad && !plan->dgrad_bf16) || (plan->fast_wgrad && !f32);
  if (need_dy && !plan->dy_direct) {
    const size_t bytes =
        static_cast<size_t>(p.batch * plan->groups * p.output_volume) * plan->dy_pad * es;
    plan->dy_pack = take(&cursor, bytes);
    if (plan->split3) plan->dy_pack_small = take(&cursor, bytes);
  }
  if ((plan->fast_dgrad || plan->fast_wgrad) && mask[2]) {
    // Upper bound of the partial count (the generic pack uses the smallest blocks).
    const size_t blocks = static_cast<size_t>((p.output_volume + 63) / 64);
    plan->bias_partial = take(&cursor, static_cast<size_t>(p.batch * plan->groups) * blocks *
                                           plan->cout_g * sizeof(float));
    plan->bias_chunks = take(&cursor, bias_chunk_bytes(static_cast<int>(plan->groups),
                                                       static_cast<int>(plan->cout_g)));
  }
  if (plan->fast_dgrad && plan->nphase > 0) {
    const size_t wes = plan->dgrad_bf16 ? 2 : es;
    for (int i = 0; i < plan->nphase; ++i) {
      int64_t sub = 1;
      for (int a = 0; a < plan->phase[i].rank; ++a) sub *= plan->phase[i].k[a];
      const size_t bytes = static_cast<size_t>(plan->groups * sub * plan->phase[i].n_pad *
                                               plan->phase[i].c_pad) * wes;
      plan->w_phase[i] = take(&cursor, bytes);
      if (plan->split3 || plan->dgrad_bf16) plan->w_phase_small[i] = take(&cursor, bytes);
    }
  } else if (plan->fast_dgrad) {
    const size_t bytes =
        static_cast<size_t>(plan->groups * taps * plan->dgrad.n_pad * plan->dgrad.c_pad) * es;
    plan->w_dg = take(&cursor, bytes);
    if (plan->split3) plan->w_dg_small = take(&cursor, bytes);
  }
  if (plan->fast_wgrad) {
    const size_t wes = f32 ? 2 : es;
    const size_t act =
        static_cast<size_t>(p.batch * plan->groups * plan->wg_x_spatial) * plan->wg_x_pad * wes;
    if (f32 || !plan->x_direct || plan->wg_fold > 1) {
      for (int part = 0; part < plan->wg_parts; ++part) plan->wg_x[part] = take(&cursor, act);
    }
    plan->partial = take(&cursor, static_cast<size_t>(plan->wgrad.splits) * plan->groups * taps *
                                      plan->cin_g * plan->cout_g * sizeof(float));
  }
  if (f32 && (plan->fast_wgrad || plan->dgrad_bf16)) {
    // dy as bfloat16 hi + lo parts, read by the weight gradient and a bf16-part dgrad
    const size_t grad =
        static_cast<size_t>(p.batch * plan->groups * p.output_volume) * plan->wg_dy_pad * 2;
    for (int part = 0; part < 2; ++part) plan->wg_dy[part] = take(&cursor, grad);
  }
  if (plan->act != 0 && ((mask[0] && !plan->fast_dgrad) || (mask[1] && !plan->fast_wgrad) ||
                         (mask[2] && !plan->fast_dgrad && !plan->fast_wgrad))) {
    plan->dz_raw = take(&cursor, static_cast<size_t>(p.batch * p.output_channels *
                                                     p.output_volume) * es);
  }
  plan->total = cursor;
}

void* at(void* base, const Region& r) {
  return r.bytes == 0 ? nullptr : static_cast<char*>(base) + r.offset;
}

int check_cuda(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return CND_OK;
}

}  // namespace
// Plans depend only on the problem (all of its bytes, which include the layout and
// activation bits and the fp32 mode), the pass kind and the gradient mask, so the host
// cost-model search runs once per distinct problem and is kept (the newest
// kPlanCacheSize problems; a shared pointer keeps a dropped plan alive for a caller still
// using it). A training step then spends no host time planning.
constexpr size_t kPlanCacheSize = 64;
struct PlanCacheEntry {
  uint64_t hash;
  int kind;
  cnd_problem problem;
  std::shared_ptr<const Plan> plan;
};
std::mutex g_plan_cache_mutex;
std::vector<PlanCacheEntry> g_plan_cache;

uint64_t problem_hash(const cnd_problem& p, int kind) {
  const unsigned char* bytes = reinterpret_cast<const unsigned char*>(&p);
  uint64_t h = 1469598103934665603ull ^ static_cast<uint64_t>(kind);
  for (size_t i = 0; i < sizeof(p); i += 8) {
    uint64_t word = 0;
    std::memcpy(&word, bytes + i, sizeof(p) - i < 8 ? sizeof(p) - i : 8);
    h = (h ^ word) * 1099511628211ull;
  }
  return h;
}

std::shared_ptr<const Plan> cached_plan(const cnd_problem& p, bool forward, const int32_t* mask) {
  const int kind =
      forward ? 8 : ((mask[0] != 0 ? 1 : 0) | (mask[1] != 0 ? 2 : 0) | (mask[2] != 0 ? 4 : 0));
  const uint64_t hash = problem_hash(p, kind);
  {
    std::lock_guard<std::mutex> lock(g_plan_cache_mutex);
    for (auto it = g_plan_cache.rbegin(); it != g_plan_cache.rend(); ++it) {
      if (it->hash == hash && it->kind == kind &&
          std::memcmp(&it->problem, &p, sizeof(p)) == 0) {
        return it->plan;
      }
    }
  }
  auto plan = std::make_shared<Plan>();
  make_plan(p, forward, mask, plan.get());
  std::lock_guard<std::mutex> lock(g_plan_cache_mutex);
  if (g_plan_cache.size() >= kPlanCacheSize) g_plan_cache.erase(g_plan_cache.begin());
  g_plan_cache.push_back(PlanCacheEntry{hash, kind, p, plan});
  return plan;
}

}  // namespace cnd

extern "C" {

size_t cnd_forward_workspace_size(const cnd_problem* problem) {
  if (problem == nullptr) return 0;
  return cnd::cached_plan(*problem, true, nullptr)->total;
}

size_t cnd_backward_workspace_size(const cnd_problem* problem, const int32_t output_mask[3]) {
  if (problem == nullptr || output_mask == nullptr) return 0;
  return cnd::cached_plan(*problem, false, output_mask)->total;
}

int cnd_fast_path_mask(const cnd_problem* problem) {
  if (problem == nullptr) return 0;
  cnd::Plan fwd, bwd;
  const int32_t all[3] = {1, 1, 1};
  cnd::make_plan(*problem, true, nullptr, &fwd);
  cnd::make_plan(*problem, false, all, &bwd);
  return (fwd.fast_fwd ? 1 : 0) | (bwd.fast_dgrad ? 2 : 0) | (bwd.fast_wgrad ? 4 : 0);
}

int cnd_plan_summary(const cnd_problem* problem, char* buffer, size_t size) {
  if (problem == nullptr) return 0;
  cnd::Plan fwd, bwd;
  const int32_t all[3] = {1, 1, 1};
  cnd::make_plan(*problem, true, nullptr, &fwd);
  cnd::make_plan(*problem, false, all, &bwd);
  char text[4096];
  int used = 0;
  auto describe = [&](const char* name, bool fast, const cnd::FpropPlan& plan,
                      const cnd::ConvPass& pass) {
    const cnd::FpropParams& P = plan.params;
    if (!fast) {
      used += std::snprintf(text + used, sizeof(text) - used, "%s: generic CUDA cores\n", name);
      return;
    }
    used += std::snprintf(text + used, sizeof(text) - used, "%s: axes [", name);
    for (int a = 0; a < pass.rank; ++a) {
      used += std::snprintf(text + used, sizeof(text) - used, a ? ",%lld" : "%lld",
                            static_cast<long long>(pass.out[a]));
    }
    used += std::snprintf(text + used, sizeof(text) - used,
                          "] tcgen05 tile [%d,%d,%d] x%d halo(a0=%d,a1=%d) box %dx%dx%d "
                          "units=%d cblocks=%d N=%d stages=%d stage_bytes=%u nacc=%d parts=%d "
                          "supers=%lld fold=%d k2f=%d tma_store=%d\n",
                          P.e0, P.b1, P.b2, P.mt, P.nshift0, P.nshift1, P.h0, P.h1, P.b2,
                          P.units, P.cblocks, P.n_pad, P.stages, P.stage_bytes, P.nacc,
                          plan.parts, static_cast<long long>(P.supers_total), P.fold,
                          P.k2f, P.tma_store);
  };
  if (bwd.bd > 1) {
    used += std::snprintf(text + used, sizeof(text) - used,
                          "groups: %d run dense (block-diagonal weights)\n", bwd.bd);
  }
  describe("forward", fwd.fast_fwd, fwd.fwd_plan, fwd.fwd);
  if (bwd.fast_dgrad && bwd.nphase > 0) {
    used += std::snprintf(text + used, sizeof(text) - used,
                          "dgrad: %d phase sub-convolutions of the strided input gradient%s\n",
                          bwd.nphase, bwd.phase_empty ? " (dx zeroed first)" : "");
    for (int i = 0; i < bwd.nphase && used < 3000; ++i) {
      char name[32];
      std::snprintf(name, sizeof(name), "dgrad phase %d", i);
      describe(name, true, bwd.phase_plan[i], bwd.phase[i]);
    }
  } else {
    describe("dgrad", bwd.fast_dgrad, bwd.dgrad_plan, bwd.dgrad);
  }
  if (bwd.fast_wgrad) {
    char detail[256];
    cnd::describe_wgrad_pass(bwd.wgrad, detail, sizeof(detail));
    used += std::snprintf(text + used, sizeof(text) - used,
                          "wgrad: tcgen05 splits=%d parts=%d taps_in_channels=%d x_pad=%lld "
                          "dy_pad=%lld %s\n",
                          bwd.wgrad.splits, bwd.wgrad.parts, bwd.wg_fold,
                          static_cast<long long>(bwd.wg_x_pad),
                          static_cast<long long>(bwd.wg_dy_pad), detail);
  } else {
    used += std::snprintf(text + used, sizeof(text) - used, "wgrad: generic CUDA cores\n");
  }
  if (buffer != nullptr && size > 0) {
    std::snprintf(buffer, size, "%s", text);
  }
  return used;
}

}  // extern "C"

namespace cnd {
namespace {

// Forward with an optional fused activation (act = 0: plain cnd_forward).
int forward_impl(const cnd_problem* problem, const void* x, const void* w, const void* b,
                 void* y, void* pre, int act, void* workspace, size_t workspace_bytes,
                 void* stream_handle) {
  clear_error();
  if (problem == nullptr || w == nullptr ||
      (problem->batch > 0 && (x == nullptr || y == nullptr))) {
    return fail(CND_ERR_INVALID, "cnd_forward: null argument");
  }
  if (act != CND_ACT_NONE && act != CND_ACT_GELU) {
    return fail(CND_ERR_UNSUPPORTED, "cnd_forward_act: unknown activation %d", act);
  }
  cnd_problem p = *problem;
  p.layout = (p.layout & 0xff) | (act << CND_LAYOUT_ACT_SHIFT);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  if (p.batch == 0) return CND_OK;
  const std::shared_ptr<const Plan> planned = cached_plan(p, true, nullptr);
  const Plan& plan = *planned;
  if (!plan.fast_fwd) {
    // generic convolution, then the activation as its own pass (pre keeps conv + b)
    void* target = (act != CND_ACT_NONE && pre != nullptr) ? pre : y;
    GenericCall call{GenericCall::kForward, &p, x, w, b, target};
    TimedPass timed(7, stream);
    int rc = run_generic(call, stream);
    if (rc != CND_OK || act == CND_ACT_NONE) return rc;
    return activation_forward(target, y, p.batch * p.output_channels * p.output_volume,
                              p.dtype, act, stream);
  }
  if (workspace_bytes < plan.total || (plan.total > 0 && workspace == nullptr)) {
    return fail(CND_ERR_WORKSPACE, "cnd_forward: workspace of %zu bytes is smaller than %zu",
                workspace_bytes, plan.total);
  }
  PackActArgs pa{};
  pa.src = x;
  pa.dst = at(workspace, plan.x_pack);
  pa.dst_small = at(workspace, plan.x_pack_small);
  pa.batch = p.batch;
  pa.groups = plan.groups;
  pa.spatial = p.input_volume;
  pa.cg = static_cast<int>(plan.cin_g);
  pa.c_pad = static_cast<int>(plan.x_pad);
  pa.dtype = p.dtype;
  pa.mode = plan.pack_mode;
  pa.chan_partial = nullptr;
  pa.src_cl = plan.x_cl ? 1 : 0;
  int rc = CND_OK;
  if (plan.x_direct) {
    pa.dst = const_cast<void*>(x);  // channels-last x is the packed operand itself
  } else {
    TimedPass timed(4, stream);
    rc = pack_activations(pa, stream);
  }
  if (rc != CND_OK) return rc;
  PackWeightArgs pw{};
  pw.w = w;
  pw.dst = at(workspace, plan.w_fwd);
  pw.dst_small = at(workspace, plan.w_fwd_small);
  pw.groups = static_cast<int>(plan.groups);
  pw.bd = plan.bd;
  pw.cout_g = static_cast<int>(plan.cout_g);
  pw.cin_g = static_cast<int>(plan.cin_g);
  pw.taps = static_cast<int>(p.kernel_volume);
  pw.n_pad = plan.fwd.n_pad;
  pw.c_pad = plan.fwd.c_pad;
  pw.dtype = p.dtype;
  pw.mode = plan.pack_mode;
  pw.dgrad = 0;
  pw.shift0 = plan.fwd_plan.shift0;
  pw.shift1 = plan.fwd_plan.shift1;
  pw.fold = plan.fwd_plan.fold;
  pw.fold2 = plan.fwd_plan.fold2;
  for (int a = 0; a < 3; ++a) pw.k_box[a] = plan.fwd_plan.k_box[a];
  {
    TimedPass timed(5, stream);
    rc = pack_weights(pw, stream);
  }
  if (rc != CND_OK) return rc;
  ConvPass pass = plan.fwd;
  pass.act = pa.dst;
  pass.act_small = pa.dst_small;
  pass.wt = pw.dst;
  pass.wt_small = pw.dst_small;
  pass.dst = y;
  pass.bias = b;
  pass.activation = act;
  pass.pre = act != CND_ACT_NONE ? pre : nullptr;
  TimedPass timed(1, stream);
  return launch_fprop(pass, plan.fwd_plan, stream, wait_timeout_ns(), 0);
}

}  // namespace
}  // namespace cnd

extern "C" {

int cnd_forward(const cnd_problem* problem, const void* x, const void* w, const void* b,
                void* y, void* workspace, size_t workspace_bytes, void* stream_handle) {
  return cnd::forward_impl(problem, x, w, b, y, nullptr, CND_ACT_NONE, workspace,
                           workspace_bytes, stream_handle);
}

int cnd_forward_act(const cnd_problem* problem, const void* x, const void* w, const void* b,
                    void* y, void* pre, int32_t activation, void* workspace,
                    size_t workspace_bytes, void* stream_handle) {
  return cnd::forward_impl(problem, x, w, b, y, pre, activation, workspace, workspace_bytes,
                           stream_handle);
}

int cnd_forward_noalloc(const cnd_problem* problem, const void* x, const void* w,
                        const void* b, void* y, void* stream_handle) {
  using namespace cnd;
  clear_error();
  if (problem == nullptr) return fail(CND_ERR_INVALID, "cnd_forward_noalloc: null argument");
  const size_t needed = cnd_forward_workspace_size(problem);
  if (needed > CND_NOALLOC_SCRATCH_BYTES) {
    return fail(CND_ERR_WORKSPACE,
                "cnd_forward_noalloc: this problem needs %zu bytes of workspace, more than "
                "the %u-byte static scratch; use cnd_forward with a caller workspace",
                needed, static_cast<unsigned>(CND_NOALLOC_SCRATCH_BYTES));
  }
  // Device address of the static scratch, looked up once per device with it current.
  static std::mutex mutex;
  static void* addresses[128] = {};
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= 128) {
    return fail(CND_ERR_CUDA, "cnd_forward_noalloc: cudaGetDevice failed");
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(mutex);
    if (addresses[device] == nullptr) {
      void* address = nullptr;
      e = cudaGetSymbolAddress(&address, g_forward_scratch);
      if (e != cudaSuccess || address == nullptr) {
        return fail(CND_ERR_CUDA, "cnd_forward_noalloc: cudaGetSymbolAddress failed: %s",
                    cudaGetErrorString(e));
      }
      addresses[device] = address;
    }
    scratch = addresses[device];
  }
  const int rc = cnd_forward(problem, x, w, b, y, needed > 0 ? scratch : nullptr, needed,
                             stream_handle);
  return rc;
}

}  // extern "C"

namespace cnd {
namespace {

// Backward with an optional fused activation backward (act = 0: plain cnd_backward).
int backward_impl(const cnd_problem* problem, const void* dy, const void* pre, int act,
                  const void* x, const void* w, void* dx, void* dw, void* db,
                  const int32_t output_mask[3], void* workspace, size_t workspace_bytes,
                  void* stream_handle) {
  clear_error();
  if (act != CND_ACT_NONE && (act != CND_ACT_GELU || (problem != nullptr &&
                                                       problem->batch > 0 && pre == nullptr))) {
    return fail(CND_ERR_INVALID, "cnd_backward_act: unknown activation or missing pre-activation");
  }
  if (problem == nullptr || output_mask == nullptr || w == nullptr) {
    return fail(CND_ERR_INVALID, "cnd_backward: null argument");
  }
  if (problem->batch > 0 && (dy == nullptr || x == nullptr)) {
    return fail(CND_ERR_INVALID, "cnd_backward: null argument");
  }
  if ((output_mask[0] && dx == nullptr && problem->batch > 0) ||
      (output_mask[1] && dw == nullptr) || (output_mask[2] && db == nullptr)) {
    return fail(CND_ERR_INVALID, "cnd_backward: missing gradient buffer");
  }
  cnd_problem p = *problem;
  p.layout = (p.layout & 0xff) | (act << CND_LAYOUT_ACT_SHIFT);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  const size_t es = element_bytes(p.dtype);
  if (p.batch == 0) {
    // Empty batch: zero parameter gradients (reference convnd.cpp:386-393).
    if (output_mask[1]) {
      cudaMemsetAsync(dw, 0,
                      static_cast<size_t>(p.output_channels * (p.channels / p.groups) *
                                          p.kernel_volume) *
                          es,
                      stream);
    }
    if (output_mask[2]) cudaMemsetAsync(db, 0, static_cast<size_t>(p.output_channels) * es, stream);
    return check_cuda("cnd_backward (empty batch)");
  }
  const std::shared_ptr<const Plan> planned = cached_plan(p, false, output_mask);
  const Plan& plan = *planned;
  if (workspace_bytes < plan.total || (plan.total > 0 && workspace == nullptr)) {
    return fail(CND_ERR_WORKSPACE, "cnd_backward: workspace of %zu bytes is smaller than %zu",
                workspace_bytes, plan.total);
  }
  int rc = CND_OK;
  const bool f32 = p.dtype == CND_F32;
  int blocks = 0;  // bias-gradient partials per (n, g), set by the pack that makes them
  float* bias_partial = static_cast<float*>(at(workspace, plan.bias_partial));
  bool bias_from_pack = false;
  // The gradient the convolution's backward sees: dy, or dy * act'(pre). It is formed by
  // the packs (pack_act / pack_pre) or, when a generic pass reads it unpacked, once in dz_raw.
  const void* grad = dy;
  int pack_act = act;
  const void* pack_pre = pre;
  if (act != CND_ACT_NONE && plan.dz_raw.bytes > 0) {
    void* dz = at(workspace, plan.dz_raw);
    rc = activation_backward(dy, pre, dz, p.batch * p.output_channels * p.output_volume,
                             p.dtype, act, stream);
    if (rc != CND_OK) return rc;
    grad = dz;
    pack_act = CND_ACT_NONE;
    pack_pre = nullptr;
  }
  const void* dy_operand = plan.dy_direct ? dy : at(workspace, plan.dy_pack);
  if (plan.dy_pack.bytes > 0 || (plan.dy_direct && output_mask[2] && bias_partial != nullptr)) {
    // dy to the packed layout, with the bias-gradient partials of the same read; when dy
    // is read in place this pass only sums its channels.
    PackActArgs pa{};
    pa.src = grad;
    pa.act = pack_act;
    pa.pre = pack_pre;
    pa.dst = at(workspace, plan.dy_pack);
    pa.dst_small = at(workspace, plan.dy_pack_small);
    pa.batch = p.batch;
    pa.groups = plan.groups;
    pa.spatial = p.output_volume;
    pa.cg = static_cast<int>(plan.cout_g);
    pa.c_pad = static_cast<int>(plan.dy_pad);
    pa.dtype = p.dtype;
    pa.mode = plan.pack_mode;
    pa.src_cl = plan.y_cl ? 1 : 0;
    pa.chan_partial = output_mask[2] ? bias_partial : nullptr;
    bias_from_pack = output_mask[2] != 0;
    if (bias_from_pack) blocks = static_cast<int>(pack_blocks(pa));
    TimedPass timed(plan.dy_direct ? 6 : 4, stream);
    rc = pack_activations(pa, stream);
    if (rc != CND_OK) return rc;
  }
  if (plan.wg_dy[0].bytes > 0) {
    // float32 dy as bfloat16 hi + lo parts (weight gradient, bf16-part dgrad)
    PackActArgs pa{};
    pa.src = grad;
    pa.act = pack_act;
    pa.pre = pack_pre;
    pa.dst = at(workspace, plan.wg_dy[0]);
    pa.dst_small = at(workspace, plan.wg_dy[1]);
    pa.batch = p.batch;
    pa.groups = plan.groups;
    pa.spatial = p.output_volume;
    pa.cg = static_cast<int>(plan.cout_g);
    pa.c_pad = static_cast<int>(plan.wg_dy_pad);
    pa.dtype = p.dtype;
    pa.mode = plan.wg_mode;
    pa.src_cl = plan.y_cl ? 1 : 0;
    if (output_mask[2] && !bias_from_pack) {
      pa.chan_partial = bias_partial;
      bias_from_pack = true;
      blocks = static_cast<int>(pack_blocks(pa));
    }
    TimedPass timed(4, stream);
    rc = pack_activations(pa, stream);
    if (rc != CND_OK) return rc;
  }
  // ---- weight gradient ----
  if (output_mask[1]) {
    if (plan.fast_wgrad) {
      WgradPass wg = plan.wgrad;
      if (plan.wg_x[0].bytes > 0) {
        PackActArgs pa{};
        pa.src = x;
        pa.dst = at(workspace, plan.wg_x[0]);
        pa.dst_small = at(workspace, plan.wg_x[1]);
        pa.dst_third = at(workspace, plan.wg_x[2]);
        pa.batch = p.batch;
        pa.groups = plan.groups;
        pa.spatial = p.input_volume;
        pa.cg = static_cast<int>(plan.cin_g);
        pa.c_pad = static_cast<int>(plan.wg_x_pad);
        pa.dtype = p.dtype;
        pa.mode = plan.wg_mode;
        pa.src_cl = plan.x_cl ? 1 : 0;
        pa.fold_taps = plan.wg_fold;
        pa.fold_dilation = static_cast<int>(plan.wg_fold_d);
        pa.fold_padding = static_cast<int>(plan.wg_fold_p);
        pa.fold_last_src = plan.wg_fold_last_src;
        pa.fold_last_dst = plan.wg_fold_last_dst;
        TimedPass timed(4, stream);
        rc = pack_activations(pa, stream);
        if (rc != CND_OK) return rc;
      }
      if (f32) {
        for (int part = 0; part < 3; ++part) wg.grad[part] = at(workspace, plan.wg_dy[part]);
      } else {
        wg.grad[0] = dy_operand;
      }
      for (int part = 0; part < 3; ++part) wg.act[part] = at(workspace, plan.wg_x[part]);
      if (plan.wg_x[0].bytes == 0) wg.act[0] = x;  // channels-last x read in place
      wg.partial = static_cast<float*>(at(workspace, plan.partial));
      {
        TimedPass timed(3, stream);
        rc = launch_wgrad_pass(wg, stream, wait_timeout_ns());
      }
      if (rc != CND_OK) return rc;
      TimedPass timed(6, stream);
      rc = reduce_wgrad(wg.partial, wg.splits, static_cast<int>(plan.groups), plan.bd,
                        static_cast<int>(p.kernel_volume), static_cast<int>(plan.cin_g),
                        static_cast<int>(plan.cout_g), dw, p.dtype, stream, plan.wg_fold);
      if (rc != CND_OK) return rc;
    } else {
      GenericCall call{GenericCall::kWgrad, &p, grad, x, nullptr, dw};
      TimedPass timed(7, stream);
      rc = run_generic(call, stream);
      if (rc != CND_OK) return rc;
    }
  }
  // ---- input gradient ----
  if (output_mask[0] && plan.fast_dgrad && plan.nphase > 0) {
    // strided: one sub-convolution per residue class of dx positions
    if (plan.phase_empty) {
      const size_t bytes =
          static_cast<size_t>(p.batch * p.channels * p.input_volume) * element_bytes(p.dtype);
      cudaMemsetAsync(dx, 0, bytes, stream);
    }
    for (int i = 0; i < plan.nphase; ++i) {
      const FpropPlan& fp = plan.phase_plan[i];
      PackWeightArgs pw = plan.phase_taps[i];
      int64_t sub = 1;
      for (int a = 0; a < plan.phase[i].rank; ++a) sub *= plan.phase[i].k[a];
      pw.w = w;
      pw.dst = at(workspace, plan.w_phase[i]);
      pw.dst_small = at(workspace, plan.w_phase_small[i]);
      pw.groups = static_cast<int>(plan.groups);
      pw.bd = plan.bd;
      pw.cout_g = static_cast<int>(plan.cout_g);
      pw.cin_g = static_cast<int>(plan.cin_g);
      pw.taps = static_cast<int>(sub);
      pw.taps_w = static_cast<int>(p.kernel_volume);
      pw.n_pad = plan.phase[i].n_pad;
      pw.c_pad = plan.phase[i].c_pad;
      pw.dtype = p.dtype;
      pw.mode = plan.dgrad_bf16 ? 4 : plan.pack_mode;
      pw.dgrad = 1;
      pw.shift0 = fp.shift0;
      pw.shift1 = fp.shift1;
      pw.fold = fp.fold;
      pw.fold2 = fp.fold2;
      for (int a = 0; a < 3; ++a) pw.k_box[a] = fp.k_box[a];
      {
        TimedPass timed(5, stream);
        rc = pack_weights(pw, stream);
      }
      if (rc != CND_OK) return rc;
      ConvPass pass = plan.phase[i];
      pass.act = plan.dgrad_bf16 ? at(workspace, plan.wg_dy[0]) : dy_operand;
      pass.act_small = at(workspace, plan.dgrad_bf16 ? plan.wg_dy[1] : plan.dy_pack_small);
      pass.wt = pw.dst;
      pass.wt_small = pw.dst_small;
      pass.dst = dx;
      pass.bias = nullptr;
      TimedPass timed(2, stream);
      rc = launch_fprop(pass, fp, stream, wait_timeout_ns(), 0);
      if (rc != CND_OK) return rc;
    }
  } else if (output_mask[0]) {
    if (plan.fast_dgrad) {
      PackWeightArgs pw{};
      pw.w = w;
      pw.dst = at(workspace, plan.w_dg);
      pw.dst_small = at(workspace, plan.w_dg_small);
      pw.groups = static_cast<int>(plan.groups);
      pw.bd = plan.bd;
      pw.cout_g = static_cast<int>(plan.cout_g);
      pw.cin_g = static_cast<int>(plan.cin_g);
      pw.taps = static_cast<int>(p.kernel_volume);
      pw.n_pad = plan.dgrad.n_pad;
      pw.c_pad = plan.dgrad.c_pad;
      pw.dtype = p.dtype;
      pw.mode = plan.dgrad_bf16 ? 4 : plan.pack_mode;
      pw.dgrad = 1;
      pw.shift0 = plan.dgrad_plan.shift0;
      pw.shift1 = plan.dgrad_plan.shift1;
      pw.fold = plan.dgrad_plan.fold;
      pw.fold2 = plan.dgrad_plan.fold2;
      for (int a = 0; a < 3; ++a) pw.k_box[a] = plan.dgrad_plan.k_box[a];
      {
        TimedPass timed(5, stream);
        rc = pack_weights(pw, stream);
      }
      if (rc != CND_OK) return rc;
      ConvPass pass = plan.dgrad;
      pass.act = plan.dgrad_bf16 ? at(workspace, plan.wg_dy[0]) : dy_operand;
      pass.act_small = at(workspace, plan.dgrad_bf16 ? plan.wg_dy[1] : plan.dy_pack_small);
      pass.wt = pw.dst;
      pass.wt_small = pw.dst_small;
      pass.dst = dx;
      pass.bias = nullptr;
      TimedPass timed(2, stream);
      rc = launch_fprop(pass, plan.dgrad_plan, stream, wait_timeout_ns(), 0);
      if (rc != CND_OK) return rc;
    } else {
      GenericCall call{GenericCall::kDgrad, &p, grad, w, nullptr, dx};
      TimedPass timed(7, stream);
      rc = run_generic(call, stream);
      if (rc != CND_OK) return rc;
    }
  }
  // ---- bias gradient ----
  if (output_mask[2]) {
    TimedPass timed(bias_from_pack ? 6 : 7, stream);
    if (bias_from_pack) {
      rc = reduce_bias(static_cast<const float*>(at(workspace, plan.bias_partial)), p.batch,
                       static_cast<int>(plan.groups), blocks, static_cast<int>(plan.cout_g), db,
                       p.dtype, static_cast<float*>(at(workspace, plan.bias_chunks)), stream);
    } else {
      GenericCall call{GenericCall::kBias, &p, grad, nullptr, nullptr, db};
      rc = run_generic(call, stream);
    }
    if (rc != CND_OK) return rc;
  }
  return CND_OK;
}

}  // namespace
}  // namespace cnd

extern "C" {

int cnd_backward(const cnd_problem* problem, const void* dy, const void* x, const void* w,
                 void* dx, void* dw, void* db, const int32_t output_mask[3], void* workspace,
                 size_t workspace_bytes, void* stream_handle) {
  return cnd::backward_impl(problem, dy, nullptr, CND_ACT_NONE, x, w, dx, dw, db, output_mask,
                            workspace, workspace_bytes, stream_handle);
}

int cnd_backward_act(const cnd_problem* problem, const void* dy, const void* pre,
                     int32_t activation, const void* x, const void* w, void* dx, void* dw,
                     void* db, const int32_t output_mask[3], void* workspace,
                     size_t workspace_bytes, void* stream_handle) {
  return cnd::backward_impl(problem, dy, pre, activation, x, w, dx, dw, db, output_mask,
                            workspace, workspace_bytes, stream_handle);
}

int cnd_device_status(void* stream_handle) {
  using namespace cnd;
  clear_error();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "cudaStreamSynchronize: %s", cudaGetErrorString(e));
  unsigned int* word = device_error_word();
  if (word == nullptr) return fail(CND_ERR_CUDA, "device error word unavailable");
  unsigned int value = 0;
  e = cudaMemcpy(&value, word, sizeof(value), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "reading the device error word: %s", cudaGetErrorString(e));
  if (value != 0) {
    cudaMemset(word, 0, sizeof(value));
    return fail(CND_ERR_TIMEOUT,
                "a bounded wait expired inside a convolution kernel (site 0x%x); results of "
                "that launch are invalid",
                value);
  }
  return CND_OK;
}

int cnd_set_kernel_timing(int32_t enable) {
  std::lock_guard<std::mutex> lock(cnd::g_timing_mutex);
  const int previous = cnd::g_timing ? 1 : 0;
  cnd::g_timing = enable != 0;
  return previous;
}

int cnd_collect_kernel_timings(int32_t* kinds, float* milliseconds, int32_t capacity) {
  std::vector<cnd::TimingRecord> records;
  {
    std::lock_guard<std::mutex> lock(cnd::g_timing_mutex);
    records.swap(cnd::g_timings);
  }
  int written = 0;
  for (const auto& r : records) {
    float ms = -1.0f;
    if (cudaEventSynchronize(r.stop) == cudaSuccess) cudaEventElapsedTime(&ms, r.start, r.stop);
    if (written < capacity && kinds != nullptr && milliseconds != nullptr) {
      kinds[written] = r.kind;
      milliseconds[written] = ms;
      ++written;
    }
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  return written;
}

int64_t cnd_launch_count(int32_t reset) {
  return reset ? cnd::g_launches.exchange(0) : cnd::g_launches.load();
}

int cnd_debug_stall_test(int32_t timeout_ms, void* stream_handle) {
  using namespace cnd;
  clear_error();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  // A 1x16x8x8 bf16 forward whose producer never issues a load: the MMA thread's bounded
  // wait on the first stage expires and the kernel returns with the error word set.
  ConvPass pass{};
  pass.rank = 2;
  pass.batch = 1;
  pass.groups = 1;
  pass.in[0] = pass.out[0] = 8;
  pass.in[1] = pass.out[1] = 16;
  pass.k[0] = pass.k[1] = 1;
  pass.s[0] = pass.s[1] = 1;
  pass.d[0] = pass.d[1] = 1;
  pass.p[0] = pass.p[1] = 0;
  pass.c_pad = 16;
  pass.n_real = 16;
  pass.n_pad = 16;
  pass.op = kOpBF16;
  pass.out_dtype = CND_BF16;
  void* buffer = nullptr;
  const size_t act = 8 * 16 * 16 * 2, wts = 16 * 16 * 2, out = 16 * 8 * 16 * 2;
  if (cudaMalloc(&buffer, 3 * 4096 + act + wts + out) != cudaSuccess) {
    return fail(CND_ERR_CUDA, "cnd_debug_stall_test: allocation failed");
  }
  char* base = static_cast<char*>(buffer);
  cudaMemsetAsync(buffer, 0, 3 * 4096 + act + wts + out, stream);
  pass.act = base;
  pass.wt = base + align_up(act);
  pass.dst = base + align_up(act) + align_up(wts);
  FpropPlan plan;
  if (!plan_fprop(pass, &plan)) {
    cudaFree(buffer);
    return fail(CND_ERR_UNSUPPORTED, "cnd_debug_stall_test: planning failed");
  }
  int rc = launch_fprop(pass, plan, stream,
                        static_cast<uint64_t>(timeout_ms > 0 ? timeout_ms : 50) * 1000000ull, 1);
  if (rc == CND_OK) rc = cnd_device_status(stream);
  cudaStreamSynchronize(stream);
  cudaFree(buffer);
  return rc;
}

}  // extern "C"
