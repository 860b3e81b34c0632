// C ABI of the tensor-product plans and launches (declared in include/ictc_cuda.h).
#include "tp_kernels.cuh"
#include "ictc_cuda.h"

#include <cstdio>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

namespace ictc {
std::vector<Variant> standalone_variants();
std::vector<Variant> message_variants();

static const std::vector<Variant>& variants() {
  static const std::vector<Variant> table = [] {
    std::vector<Variant> all = standalone_variants();
    std::vector<Variant> msg = message_variants();
    all.insert(all.end(), msg.begin(), msg.end());
    return all;
  }();
  return table;
}

static const Variant* find_variant(int li, int le, int lo, int cpl, int layout, int kind) {
  for (const Variant& v : variants())
    if (v.li == li && v.le == le && v.lo == lo && v.cpl == cpl && v.layout == layout && v.kind == kind) return &v;
  return nullptr;
}
}  // namespace ictc

using namespace ictc;

struct ictc_tp_plan {
  int channels, li, le, lo, layout;
  const Variant* v[kKinds];
  int cpl[kKinds], slices[kKinds], block[kKinds], grid[kKinds];
  size_t smem[kKinds];
  int stage_floats;         // graph adjoint staging buffer per warp (0 = not staged)
  size_t adj_staged_smem;
  int adj_staged_grid;
  // Staged graph forward, two channels per lane (one warp per node), used when
  // the feature and gate rows of a launch are 16-byte aligned; else v[kMessageForward].
  const Variant* fwd2;
  int fwd2_stage_floats, fwd2_grid;
  size_t fwd2_smem;
  std::vector<float> coef;  // host copy of the dense CG table (kernel-parameter source)
  float* d_coef;
  int2* d_desc;
  int* d_status;            // non-zero after a kernel gave up on a timed-out wait
  int device;
};

static thread_local char g_error[512] = "";

void ictc_set_error(const char* fmt, const char* detail) {
  snprintf(g_error, sizeof(g_error), fmt, detail ? detail : "");
}

extern "C" const char* ictc_last_error(void) { return g_error; }

extern "C" int ictc_version(void) { return ICTC_ABI_VERSION; }

// Largest instantiated channels-per-lane <= preferred that divides C, keeps
// every slice but the last full, and (for grouped kinds) needs <= 8 slices.
static int pick_cpl(int li, int le, int lo, int layout, int kind, int channels, int preferred) {
  for (int cpl = preferred; cpl >= 1; cpl /= 2) {
    if (channels % cpl) continue;
    if (cpl > 1 && channels < 32 * cpl) continue;
    int slices = (channels + 32 * cpl - 1) / (32 * cpl);
    if ((kind == kAdjoint || kind == kMessageAdjoint) && slices > kWarps) continue;
    if (find_variant(li, le, lo, cpl, layout, kind)) return cpl;
  }
  return 0;
}

extern "C" int ictc_tp_plan_create(int channels, int input_lmax, int edge_lmax, int output_lmax, int layout,
                                   int num_paths, const int32_t* paths, const double* cg, int64_t cg_len,
                                   int cpl_forward, int cpl_backward, ictc_tp_plan** out) {
  if (!out || !paths || !cg) {
    ictc_set_error("ictc_tp_plan_create: invalid (null) argument%s", "");
    return ICTC_ERR_INVALID;
  }
  *out = nullptr;
  if (layout != kIrMul && layout != kMulIr) {
    ictc_set_error("ictc_tp_plan_create: invalid layout, must be 0 (ir_mul) or 1 (mul_ir)%s", "");
    return ICTC_ERR_INVALID;
  }
  if (channels <= 0 || input_lmax < 0 || edge_lmax < 0 || output_lmax < 0 || input_lmax > 6 || edge_lmax > 6 ||
      output_lmax > 6) {
    ictc_set_error("ictc_tp_plan_create: invalid channel count or degree%s", "");
    return ICTC_ERR_INVALID;
  }
  const PathTable ref = make_paths(input_lmax, edge_lmax, output_lmax);
  if (num_paths != ref.np) {
    ictc_set_error("ictc_tp_plan_create: path list does not match the operator path set%s", "");
    return ICTC_ERR_UNSUPPORTED;
  }
  int64_t expect = 0;
  for (int p = 0; p < num_paths; ++p) {
    if (paths[3 * p] != ref.l1[p] || paths[3 * p + 1] != ref.l2[p] || paths[3 * p + 2] != ref.l3[p]) {
      ictc_set_error("ictc_tp_plan_create: path order differs from the operator path order%s", "");
      return ICTC_ERR_UNSUPPORTED;
    }
    expect += (2 * ref.l1[p] + 1) * (2 * ref.l2[p] + 1) * (2 * ref.l3[p] + 1);
  }
  if (cg_len != expect) {
    ictc_set_error("ictc_tp_plan_create: invalid CG buffer length%s", "");
    return ICTC_ERR_INVALID;
  }
  ictc_tp_plan* plan = new (std::nothrow) ictc_tp_plan();
  if (!plan) return ICTC_ERR_NOMEM;
  plan->channels = channels; plan->li = input_lmax; plan->le = edge_lmax; plan->lo = output_lmax;
  plan->layout = layout;
  const int rows = ref.out_rows;
  const int preferred[kKinds] = {cpl_forward > 0 ? cpl_forward : 4, cpl_backward > 0 ? cpl_backward : 2,
                                 1, cpl_backward > 0 ? cpl_backward : 2};
  for (int kind = 0; kind < kKinds; ++kind) {
    int cpl = pick_cpl(input_lmax, edge_lmax, output_lmax, layout, kind, channels, preferred[kind]);
    plan->v[kind] = cpl ? find_variant(input_lmax, edge_lmax, output_lmax, cpl, layout, kind) : nullptr;
    if (!plan->v[kind]) {
      delete plan;
      ictc_set_error("ictc_tp_plan_create: no kernel for this degree set / channel count%s", "");
      return ICTC_ERR_UNSUPPORTED;
    }
    plan->cpl[kind] = cpl;
    plan->slices[kind] = (channels + 32 * cpl - 1) / (32 * cpl);
    plan->smem[kind] = plan->v[kind]->smem;
    plan->block[kind] = (kind == kAdjoint || kind == kMessageAdjoint)
                            ? 32 * plan->slices[kind] * (kWarps / plan->slices[kind])
                            : kThreads;
  }
  // The kernels skip structurally zero CG terms of the frozen ICTC basis at
  // compile time; reject a CG table with a significant entry outside that pattern.
  {
    int64_t off = 0;
    for (int p = 0; p < num_paths; ++p) {
      int l1 = ref.l1[p], l2 = ref.l2[p], l3 = ref.l3[p];
      int m1 = 2 * l1 + 1, m2 = 2 * l2 + 1, m3 = 2 * l3 + 1;
      double peak = 0.0;
      for (int t = 0; t < m1 * m2 * m3; ++t) peak = fmax(peak, fabs(cg[off + t]));
      for (int i = 0; i < m1; ++i)
        for (int j = 0; j < m2; ++j)
          for (int k = 0; k < m3; ++k)
            if (!cg_nonzero(l1, l2, l3, i, j, k) && fabs(cg[off + (i * m2 + j) * m3 + k]) > 1e-10 * peak) {
              delete plan;
              ictc_set_error("ictc_tp_plan_create: CG tensors are not in the frozen ICTC basis pattern%s", "");
              return ICTC_ERR_UNSUPPORTED;
            }
      off += (int64_t)m1 * m2 * m3;
    }
  }
  // Re-lay the per-path CG tensors C_p[i][j][k] as [p][i][k][j] and build the
  // bond column descriptors.
  std::vector<float> coef(ref.coef_total);
  std::vector<int2> desc(ref.bond_width);
  int64_t src = 0;
  for (int p = 0; p < num_paths; ++p) {
    int m1 = 2 * ref.l1[p] + 1, m2 = 2 * ref.l2[p] + 1, m3 = 2 * ref.l3[p] + 1;
    for (int i = 0; i < m1; ++i)
      for (int j = 0; j < m2; ++j)
        for (int k = 0; k < m3; ++k)
          coef[ref.coef_off[p] + (i * m3 + k) * m2 + j] = (float)cg[src + (i * m2 + j) * m3 + k];
    for (int i = 0; i < m1; ++i)
      for (int k = 0; k < m3; ++k) {
        int col = ref.bond_off[p] + i * m3 + k;
        desc[col].x = (ref.l2[p] * ref.l2[p]) | (m2 << 16);
        desc[col].y = ref.coef_off[p] + (i * m3 + k) * m2;
      }
    src += (int64_t)m1 * m2 * m3;
  }
  // The graph adjoint stages each edge's output-gradient and gate rows in shared
  // memory when a node is one warp and the rows are whole 16-byte units that fit.
  {
    const Variant* va = plan->v[kMessageAdjoint];
    const int stage = (va->rows + va->np) * channels;
    const bool fits = va->fn_staged && plan->slices[kMessageAdjoint] == 1 && (va->rows * channels) % 4 == 0 &&
                      (va->np * channels) % 4 == 0 && stage * 4 <= kStageBudgetBytes;
    plan->stage_floats = fits ? stage : 0;
    plan->adj_staged_smem = fits ? staged_smem_bytes((int)va->smem, stage) : 0;
    plan->adj_staged_grid = 0;
  }
  plan->fwd2 = nullptr;
  plan->fwd2_stage_floats = plan->fwd2_grid = 0;
  plan->fwd2_smem = 0;
  if (channels == 64) {
    const Variant* v2 = find_variant(input_lmax, edge_lmax, output_lmax, 2, layout, kMessageForward);
    if (v2 && (v2->a * channels) % 4 == 0 && (v2->np * channels) % 4 == 0 &&
        2 * (v2->a + v2->np) * channels * 4 <= 2 * kStageBudgetBytes) {
      plan->fwd2 = v2;
      plan->fwd2_stage_floats = (v2->a + v2->np) * channels;
      plan->fwd2_smem = staged_smem_bytes((int)v2->smem, 2 * plan->fwd2_stage_floats);
    }
  }
  plan->coef = coef;
  cudaGetDevice(&plan->device);
  plan->d_coef = nullptr;
  plan->d_desc = nullptr;
  plan->d_status = nullptr;
  if (cudaMalloc(&plan->d_coef, sizeof(float) * (coef.size() + 4)) != cudaSuccess ||
      cudaMalloc(&plan->d_desc, sizeof(int2) * (desc.size() + 4)) != cudaSuccess ||
      cudaMalloc(&plan->d_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(plan->d_coef);
    cudaFree(plan->d_desc);
    delete plan;
    ictc_set_error("ictc_tp_plan_create: device allocation failed%s", "");
    return ICTC_ERR_NOMEM;
  }
  cudaMemcpy(plan->d_coef, coef.data(), sizeof(float) * coef.size(), cudaMemcpyHostToDevice);
  cudaMemcpy(plan->d_desc, desc.data(), sizeof(int2) * desc.size(), cudaMemcpyHostToDevice);
  cudaMemset(plan->d_status, 0, sizeof(int));
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, plan->device);
  for (int kind = 0; kind < kKinds; ++kind) {
    const Variant* v = plan->v[kind];
    int per_sm = 0;
    cudaFuncSetAttribute(v->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan->smem[kind]);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, v->fn, plan->block[kind], plan->smem[kind]);
    plan->grid[kind] = sms * (per_sm < 1 ? 1 : per_sm);
  }
  if (plan->stage_floats > 0) {
    const Variant* va = plan->v[kMessageAdjoint];
    int per_sm = 0;
    cudaFuncSetAttribute(va->fn_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan->adj_staged_smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, va->fn_staged, plan->block[kMessageAdjoint],
                                                  plan->adj_staged_smem);
    plan->adj_staged_grid = sms * (per_sm < 1 ? 1 : per_sm);
  }
  if (plan->fwd2) {
    int per_sm = 0;
    cudaFuncSetAttribute(plan->fwd2->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan->fwd2_smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plan->fwd2->fn, kThreads, plan->fwd2_smem);
    plan->fwd2_grid = sms * (per_sm < 1 ? 1 : per_sm);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    ictc_set_error("ictc_tp_plan_create: %s", cudaGetErrorString(err));
    cudaFree(plan->d_coef);
    cudaFree(plan->d_desc);
    cudaFree(plan->d_status);
    delete plan;
    return ICTC_ERR_CUDA;
  }
  *out = plan;
  return ICTC_OK;
}

extern "C" int ictc_tp_plan_destroy(ictc_tp_plan* plan) {
  if (!plan) return ICTC_OK;
  cudaFree(plan->d_coef);
  cudaFree(plan->d_desc);
  cudaFree(plan->d_status);
  delete plan;
  return ICTC_OK;
}

extern "C" int ictc_tp_plan_status(const ictc_tp_plan* plan, int32_t* status, int reset) {
  if (!plan || !status) {
    ictc_set_error("ictc_tp_plan_status: invalid (null) argument%s", "");
    return ICTC_ERR_INVALID;
  }
  int value = 0;
  cudaError_t err = cudaMemcpy(&value, plan->d_status, sizeof(int), cudaMemcpyDeviceToHost);
  if (err == cudaSuccess && reset) err = cudaMemset(plan->d_status, 0, sizeof(int));
  if (err != cudaSuccess) {
    ictc_set_error("ictc_tp_plan_status: %s", cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  *status = value;
  return ICTC_OK;
}

extern "C" int ictc_tp_plan_info(const ictc_tp_plan* plan, int64_t* info, int n) {
  if (!plan || !info) {
    ictc_set_error("ictc_tp_plan_info: invalid (null) argument%s", "");
    return ICTC_ERR_INVALID;
  }
  const Variant* v = plan->v[kForward];
  int64_t values[12] = {v->np, v->bond_width, v->rows * (int64_t)plan->channels, v->a * (int64_t)plan->channels,
                        v->b, plan->cpl[kForward], plan->cpl[kAdjoint], plan->grid[kForward],
                        plan->cpl[kMessageForward], plan->cpl[kMessageAdjoint], plan->grid[kAdjoint],
                        plan->block[kAdjoint]};
  for (int t = 0; t < n && t < 12; ++t) info[t] = values[t];
  return ICTC_OK;
}

static int launch(const ictc_tp_plan* plan, int kind, TPArgs& args, int64_t units_per_block, void* stream,
                  const char* what) {
  args.coef = plan->d_coef;
  args.desc = plan->d_desc;
  args.channels = plan->channels;
  args.slices = plan->slices[kind];
  args.status = plan->d_status;
  args.stage_floats = 0;
  const Variant* v = plan->v[kind];
  int grid_cap = plan->grid[kind];
  size_t smem = plan->smem[kind];
  if (kind == kMessageForward && plan->fwd2 && (reinterpret_cast<uintptr_t>(args.features) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(args.gates) & 15u) == 0) {
    v = plan->fwd2;
    grid_cap = plan->fwd2_grid;
    smem = plan->fwd2_smem;
    args.slices = 1;
    args.stage_floats = plan->fwd2_stage_floats;
  }
  Launcher launcher = v->launch;
  if (kind == kMessageAdjoint && plan->stage_floats > 0 &&
      (reinterpret_cast<uintptr_t>(args.grad_out) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(args.gates) & 15u) == 0) {
    args.stage_floats = plan->stage_floats;
    launcher = v->launch_staged;
    grid_cap = plan->adj_staged_grid;
    smem = plan->adj_staged_smem;
  }
  if (args.rows <= 0) return ICTC_OK;
  int64_t work = (args.rows * (kind == kAdjoint || kind == kMessageAdjoint ? 1 : args.slices) + units_per_block - 1) /
                 units_per_block;
  int grid = (int)(work < grid_cap ? work : grid_cap);
  cudaError_t err = launcher(args, plan->coef.data(), grid, plan->block[kind], smem, (cudaStream_t)stream);
  if (err != cudaSuccess) {
    ictc_set_error(what, cudaGetErrorString(err));
    return ICTC_ERR_CUDA;
  }
  return ICTC_OK;
}

extern "C" int ictc_tp_forward(const ictc_tp_plan* plan, const float* features, const float* harmonics,
                               const float* gates, const float* weight, float* out, int64_t rows,
                               void* stream) {
  if (!plan || rows < 0 || (rows > 0 && (!features || !harmonics || !out))) {
    ictc_set_error("ictc_tp_forward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  TPArgs a{};
  a.features = features; a.harmonics = harmonics; a.gates = gates; a.weight = weight; a.out = out;
  a.rows = rows;
  return launch(plan, kForward, a, kWarps, stream, "tensor-product forward launch failed: %s");
}

extern "C" int ictc_tp_backward(const ictc_tp_plan* plan, const float* features, const float* harmonics,
                                const float* gates, const float* weight, const float* grad_out,
                                float* grad_features, float* grad_harmonics, float* grad_gates, int64_t rows,
                                void* stream) {
  if (!plan || rows < 0 || (rows > 0 && (!features || !harmonics || !grad_out))) {
    ictc_set_error("ictc_tp_backward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  TPArgs a{};
  a.features = features; a.harmonics = harmonics; a.gates = gates; a.weight = weight; a.grad_out = grad_out;
  a.grad_features = grad_features; a.grad_harmonics = grad_harmonics; a.grad_gates = grad_gates;
  a.rows = rows;
  int groups = plan->block[kAdjoint] / 32 / plan->slices[kAdjoint];
  return launch(plan, kAdjoint, a, groups, stream, "tensor-product adjoint launch failed: %s");
}

extern "C" int ictc_tp_message_forward(const ictc_tp_plan* plan, const float* node_features,
                                       const float* harmonics, const float* gates, const float* weight,
                                       const float* mask, const int64_t* src, const int64_t* dst_order,
                                       const int64_t* dst_offsets, float* out, int64_t dst_nodes, void* stream) {
  if (!plan || dst_nodes < 0 ||
      (dst_nodes > 0 && (!node_features || !harmonics || !src || !dst_offsets || !out))) {
    ictc_set_error("ictc_tp_message_forward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  TPArgs a{};
  a.features = node_features; a.harmonics = harmonics; a.gates = gates; a.weight = weight; a.mask = mask;
  a.src = src; a.order = dst_order; a.offsets = dst_offsets; a.out = out; a.rows = dst_nodes;
  return launch(plan, kMessageForward, a, kWarps, stream, "graph-message forward launch failed: %s");
}

extern "C" int ictc_tp_message_backward(const ictc_tp_plan* plan, const float* node_features,
                                        const float* harmonics, const float* gates, const float* weight,
                                        const float* mask, const int64_t* dst, const int64_t* src_order,
                                        const int64_t* src_offsets, const float* grad_out,
                                        float* grad_node_features, float* grad_harmonics, float* grad_gates,
                                        int64_t src_nodes, void* stream) {
  if (!plan || src_nodes < 0 ||
      (src_nodes > 0 && (!node_features || !harmonics || !dst || !src_offsets || !grad_out))) {
    ictc_set_error("ictc_tp_message_backward: invalid argument%s", "");
    return ICTC_ERR_INVALID;
  }
  TPArgs a{};
  a.features = node_features; a.harmonics = harmonics; a.gates = gates; a.weight = weight; a.mask = mask;
  a.dst = dst; a.order = src_order; a.offsets = src_offsets; a.grad_out = grad_out;
  a.grad_features = grad_node_features; a.grad_harmonics = grad_harmonics; a.grad_gates = grad_gates;
  a.rows = src_nodes;
  int groups = plan->block[kMessageAdjoint] / 32 / plan->slices[kMessageAdjoint];
  return launch(plan, kMessageAdjoint, a, groups, stream, "graph-message adjoint launch failed: %s");
}
