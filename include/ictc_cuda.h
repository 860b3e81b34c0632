/*
 * ictc_cuda.h -- C ABI of libictc_cuda.so, the B200 (sm_100a) backend for the
 * ICTC-O3 hot path: the channelwise path-preserving O(3) tensor product (TP),
 * its adjoints, and the direction harmonics that feed it.
 *
 * Conventions
 *   - Plain C: pointers, sizes, status codes.  No torch or CUDA types; a
 *     `stream` argument is a cudaStream_t passed as void* (NULL = legacy
 *     default stream).  Every launch is asynchronous on that stream.
 *   - All tensors are row-major, contiguous, FP32 device memory.  The caller
 *     owns every buffer; entry points allocate nothing except inside
 *     ictc_tp_plan_create (the plan's constant tables).
 *   - Packed layouts follow the reference's public operator
 *     (ictc_o3/operators.py:77-127):
 *       features  [rows, C*(Li+1)^2]  degree-major; inside degree l either
 *                 ir_mul = [2l+1][C] (layout 0) or mul_ir = [C][2l+1] (layout 1)
 *       harmonics [rows, (Le+1)^2]    Y_0 | Y_1 | ... (ictc_o3/operators.py:101-105)
 *       gates     [rows, P*C]         path-major, channel-minor, or NULL
 *       weight    [P, C]              per-(path, channel) weight, or NULL (= 1)
 *       out       [rows, C*sum_l count_l*(2l+1)]  ordered by l3, then path
 *                 offset, then the same inner layout (ictc_o3/operators.py:107-127)
 *   - Return value: ICTC_OK (0) or a negative ICTC_ERR_*; ictc_last_error()
 *     returns a message for the calling thread.
 */
#ifndef ICTC_CUDA_H
#define ICTC_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ICTC_ABI_VERSION 2

#define ICTC_OK 0
#define ICTC_ERR_INVALID (-1)     /* bad pointer, size or shape            */
#define ICTC_ERR_UNSUPPORTED (-2) /* no kernel for this degree/channel set */
#define ICTC_ERR_CUDA (-3)        /* CUDA launch or runtime error          */
#define ICTC_ERR_NOMEM (-4)       /* device or host allocation failed      */

typedef struct ictc_tp_plan ictc_tp_plan;

/* ABI version compiled into the library (ICTC_ABI_VERSION). */
int ictc_version(void);

/* Message of the last error raised on the calling thread ("" if none). */
const char* ictc_last_error(void);

/*
 * Build the constant tables of one path-preserving TP on the current device.
 * Replaces the reference's cached plan construction
 * (ictc_o3/backends/ascend/tensor_product.py:9-57, `_plan`), which packs the
 * owner's CG list (`_get_cg_list`, ictc_o3/basis/ictd_irreps.py:2219-2237)
 * into sparse routing tables for the native map.
 *   paths   [num_paths][3] = (l1, l2, l3) in the owner's path order
 *   cg      concatenation of the normalised per-path CG tensors
 *           C_p[m1][m2][m3] (float64), cg_len values in total
 *   cpl_forward / cpl_backward: channels per lane (1, 2 or 4; 0 = default)
 */
int ictc_tp_plan_create(int channels, int input_lmax, int edge_lmax, int output_lmax, int layout,
                        int num_paths, const int32_t* paths, const double* cg, int64_t cg_len,
                        int cpl_forward, int cpl_backward, ictc_tp_plan** plan);

/* Release a plan (NULL is accepted). */
int ictc_tp_plan_destroy(ictc_tp_plan* plan);

/* Plan metadata (first n of): [num_paths, bond_width, output_width,
 * feature_width, harmonic_width, cpl_forward, cpl_backward, forward grid,
 * cpl_message_forward, cpl_message_backward, adjoint grid, adjoint block]. */
int ictc_tp_plan_info(const ictc_tp_plan* plan, int64_t* info, int n);

/* Status word of the plan's kernels: *status = 0, or non-zero after a kernel
 * gave up on a timed-out wait (the graph kernels' staged row copies); the
 * kernel then leaves its remaining work undone.  1: a copy did not land in
 * time and the copies in flight drained (the context stays usable); 2: a launch
 * shape the kernel does not support; 3: a copy did not land and the drain timed
 * out too, so a bulk copy may still write shared memory after its CTA ended --
 * treat the CUDA context as lost.  The word keeps the largest code.  Reads one
 * int from the device (synchronising); reset != 0 clears the word.  No
 * reference counterpart: the reference backends have no asynchronous copies to
 * lose. */
int ictc_tp_plan_status(const ictc_tp_plan* plan, int32_t* status, int reset);

/*
 * TP forward, out = TP(features, harmonics, gates * weight).
 * Replaces mode 0 of the native sparse trilinear map
 * (ictc_o3/ascendc/op_kernel/weighted_map.cpp:263 `ictc_weighted_map`, bound
 * at ictc_o3/ascendc/op_host/bindings.cpp:92 `weighted_map`) and the packed
 * GEMM schedule (ictc_o3/backends/ascend/packed_tensor_product.py:60-80).
 */
int ictc_tp_forward(const ictc_tp_plan* plan, const float* features, const float* harmonics,
                    const float* gates, const float* weight, float* out, int64_t rows, void* stream);

/*
 * Fused first-order adjoint of ictc_tp_forward for cotangent grad_out.
 * Any of grad_features / grad_harmonics / grad_gates may be NULL (not
 * computed); non-NULL outputs are fully overwritten.  With gates == NULL,
 * grad_gates receives the per-row gradient of the effective weight.
 * Replaces modes 1-3 (dL, dR, dW) of `ictc_weighted_map`
 * (ictc_o3/ascendc/op_kernel/weighted_map.cpp:263) and the recursive GEMM
 * adjoint (ictc_o3/backends/ascend/packed_tensor_product.py:82-110).
 */
int ictc_tp_backward(const ictc_tp_plan* plan, const float* features, const float* harmonics,
                     const float* gates, const float* weight, const float* grad_out,
                     float* grad_features, float* grad_harmonics, float* grad_gates, int64_t rows,
                     void* stream);

/*
 * Graph message, out[n] = sum_{e: dst_e = n} mask_e * TP(node_features[src_e],
 * harmonics_e, gates_e * weight) for n < dst_nodes, evaluated over a
 * destination-sorted CSR (dst_order: edge ids grouped by destination, or NULL
 * when the edges are already grouped by destination; dst_offsets
 * [dst_nodes+1]).  Every output row is written (zero for nodes
 * without edges); no atomics.  mask [E] may be NULL.  Indices must be valid
 * (src_e < rows of node_features, dst_e < dst_nodes); the host validates them.
 * Replaces the fused gather / TP / FP32-atomic scatter of `ictc_weighted_map`
 * in graph mode (ictc_o3/ascendc/op_kernel/weighted_map.cpp:178-233), the
 * gate-and-scatter epilogue (ictc_o3/ascendc/op_kernel/epilogue.cpp:192) and
 * the chunked message schedules (ictc_o3/ascendc/graph.py:22-76,
 * ictc_o3/backends/ascend/channel_message.py:35-216).
 */
int ictc_tp_message_forward(const ictc_tp_plan* plan, const float* node_features, const float* harmonics,
                            const float* gates, const float* weight, const float* mask, const int64_t* src,
                            const int64_t* dst_order, const int64_t* dst_offsets, float* out, int64_t dst_nodes,
                            void* stream);

/*
 * Fused first-order adjoint of ictc_tp_message_forward for cotangent grad_out
 * [dst_nodes, output_width], walked over a source-sorted CSR (src_order, or
 * NULL when the edges are already grouped by source; src_offsets [src_nodes+1]).  Writes grad_node_features [src_nodes, ...]
 * (zero rows for nodes without edges), grad_harmonics [E, B] and grad_gates
 * [E, P*C] (any may be NULL).  Replaces the epilogue adjoints
 * (ictc_o3/ascendc/op_kernel/epilogue.cpp:192 modes 1-2) and the capacity
 * first-order backward (ictc_o3/backends/ascend/capacity_adjoint.py:56-148).
 */
int ictc_tp_message_backward(const ictc_tp_plan* plan, const float* node_features, const float* harmonics,
                             const float* gates, const float* weight, const float* mask, const int64_t* dst,
                             const int64_t* src_order, const int64_t* src_offsets, const float* grad_out,
                             float* grad_node_features, float* grad_harmonics, float* grad_gates,
                             int64_t src_nodes, void* stream);

/* Number of floats in the direction-harmonic table for degrees 1..lmax:
 * sum_l Dsym(l) * (2l+1), Dsym(l) = (l+1)(l+2)/2. */
int ictc_harmonics_table_size(int lmax);

/*
 * ICTC direction harmonics of row vectors n [rows, 3] for l = 0..lmax
 * (1 <= lmax <= 6), output [rows, (lmax+1)^2] = Y_0 | Y_1 | ... .
 * table: for l = 1..lmax, H_l[d][m] (row-major, monomials in ICTC order)
 *        = multinomial_d * (G_l B_l)[d][m] * component_scale_l.
 * mode 0: out0 = Y(n)                                  (grad_y, grad_dir unused)
 * mode 1: out0[rows,3] = J(n)^T grad_y                 (first adjoint)
 * mode 2: out0[rows,W] = J(n) grad_dir,  out1[rows,3] = sum_m grad_y[m] Hess Y_m(n) grad_dir
 * Replaces the generated Triton harmonics and their analytic adjoints
 * (ictc_o3/ops/generated_direction_harmonics.py:43-177) and the reference
 * evaluation direction_harmonics_all (ictc_o3/basis/ictd_irreps.py:1113-1168).
 */
int ictc_direction_harmonics(const float* directions, const float* table, const float* grad_y,
                             const float* grad_dir, float* out0, float* out1, int64_t rows, int lmax,
                             int mode, void* stream);

/*
 * Edge geometry of one interaction, fused: for edge vectors vec [E, 3],
 *   unit = vec / max(|vec|, 1e-8)  [E, 3],  mask = (|vec| <= r_max)  [E],
 *   radial [E, num_basis] = Bessel basis sqrt(2/r_max) sin(b pi r / r_max) / r
 *                           x polynomial envelope of order p (x sqrt(num_basis) if basis_norm).
 * Replaces the elementwise chain of mace_ictc/models/radial_basis.py:11-39
 * (mace_polynomial_cutoff) and :42-91 (mace_radial_embedding, Bessel kind) with the
 * edge normalisation of the interaction's edge features.  num_basis <= 16, p >= 1.
 * The backward maps grad_unit [E, 3] and grad_radial [E, num_basis] (either may be
 * NULL) to grad_vec [E, 3].
 */
int ictc_edge_geometry(const float* vec, int64_t edges, float r_max, int num_basis, int p, int basis_norm,
                       float* unit, float* radial, float* mask, void* stream);
int ictc_edge_geometry_backward(const float* vec, const float* grad_unit, const float* grad_radial, int64_t edges,
                                float r_max, int num_basis, int p, int basis_norm, float* grad_vec, void* stream);

/*
 * MACE symmetric contraction as a per-node polynomial (correlation 1..3,
 * input degrees 0..lmax with 1 <= lmax <= 3, targets 0..target_lmax <= lmax).
 *   x      [N, C*(lmax+1)^2]   node features, degree blocks [C][2l+1] (mul_ir)
 *   table  [S, R, C]           species coefficient table T = Usym * W (ictc_sc_fold):
 *          for each target t, monomial rows in the order
 *          for i: (i); for j >= i: (i,j); for k >= j: (i,j,k)   (orders <= correlation)
 *          each row holding 2t+1 consecutive C-vectors; R = ictc_sc_table_rows(...)
 *   tiles  [num_tiles, ictc_sc_tile_nodes()] node ids of one species each, -1 padded;
 *          tile_species [num_tiles]
 *   out    [N, C*(target_lmax+1)^2]  target blocks [C][2t+1] (mul_ir)
 * Nodes not named by any tile are not written.  Replaces the MACE recursion
 * (ictc_o3/ops/_mace_symmetric_contraction.py:298-346) and the Ascend factorised
 * contraction (ictc_o3/backends/ascend/contraction.py:8-45).
 */
int64_t ictc_sc_table_rows(int lmax, int correlation, int target_lmax);
int ictc_sc_tile_nodes(void);
int ictc_sc_forward(const float* x, const float* table, const int64_t* tiles, const int32_t* tile_species,
                    int64_t num_tiles, float* out, int channels, int lmax, int correlation, int target_lmax,
                    void* stream);

/* Feature gradient of ictc_sc_forward for cotangent grad_out: grad_x [N, C*(lmax+1)^2]
 * (rows of nodes named by a tile are fully written). */
int ictc_sc_backward(const float* x, const float* table, const int64_t* tiles, const int32_t* tile_species,
                     int64_t num_tiles, const float* grad_out, float* grad_x, int channels, int lmax,
                     int correlation, int target_lmax, void* stream);

/* Weight fold of one target degree of the symmetric contraction (replaces the
 * species-bank projection of backends/ascend/contraction.py:8-45, the dense GEMM
 * that folds the weights into the coupling constants):
 *   adjoint = 0: table[s, row0 + r, c] = sum_p usym[r, p] * weights[s, p, c]
 *   adjoint = 1: weights[s, p, c] = sum_r usym[r, p] * table[s, row0 + r, c]
 *                (the weight gradient: table holds dT, weights receives dW)
 * usym [rows, cols] (symmetrised couplings, rows = monomials x (2t+1)),
 * weights [species, cols, channels], table [species, table_rows, channels].
 * The couplings may be either of the reference's parameterisations (pure-ICTC U,
 * or bridge-U with its basis bridge folded in, ictc_o3/ops/symmetric_contraction.py:92-206):
 * the kernels only see their symmetrised rows.  Deterministic (no atomics). */
int ictc_sc_fold(const float* usym, const float* weights, float* table, int rows, int cols, int channels,
                 int species, int64_t table_rows, int64_t row0, int adjoint, void* stream);

/* Second derivatives of ictc_sc_forward (force-loss training; no reference kernel:
 * the reference differentiates its recursion with autograd,
 * ictc_o3/backends/ascend/sparse_product.py:226-264).  dir [N, C*(lmax+1)^2] is a
 * direction h in feature space; with the directional monomials (h.grad) mono(x):
 *   ictc_sc_directional: out[n] = sum_r T[r] (h.grad) mono_r(x)  (derivative of the
 *                        feature gradient with respect to the output cotangent)
 *   ictc_sc_hvp:         grad_x[n] = gradient in x of sum_m grad_out[m] (h.grad) out[m]
 *                        (Hessian-vector product of the polynomial)
 *   ictc_sc_table_grad:  grad_table[s, row, c] = sum_{n of species s} grad_out[n] * v_row(n)
 *                        with v = mono(x), or (h.grad) mono(x) when dir != NULL;
 *                        tiles must list the species in ascending order (as the host
 *                        builds them); every [species, row, channel] entry is written.
 * Deterministic (no atomics). */
int ictc_sc_directional(const float* x, const float* dir, const float* table, const int64_t* tiles,
                        const int32_t* tile_species, int64_t num_tiles, float* out, int channels, int lmax,
                        int correlation, int target_lmax, void* stream);
int ictc_sc_hvp(const float* x, const float* dir, const float* table, const int64_t* tiles,
                const int32_t* tile_species, int64_t num_tiles, const float* grad_out, float* grad_x, int channels,
                int lmax, int correlation, int target_lmax, void* stream);
int ictc_sc_table_grad(const float* x, const float* dir, const float* grad_out, const int64_t* tiles,
                       const int32_t* tile_species, int64_t num_tiles, float* grad_table, int species, int channels,
                       int lmax, int correlation, int target_lmax, void* stream);

/*
 * Periodic cell-list neighbour search (orthorhombic box, cutoff < L/2, >= 3
 * cells per axis).  Produces the destination-sorted edge list of the message
 * kernels: for receiver i, neighbours j with |pos[i] - pos[j] + shift| < cutoff
 * (minimum image), grouped by i and ordered by neighbour cell then atom id.
 * Replaces the torch-only radius graph (mace_ictc/utils/graph_utils.py:217-297).
 *   box: host pointer to the three box lengths.
 *   workspace: device scratch of ictc_neighbor_workspace_bytes(...) bytes, owned
 *   by the caller; ictc_neighbor_fill must get the workspace that the preceding
 *   ictc_neighbor_count on the same stream filled.
 *   ictc_neighbor_count writes offsets [atoms + 1] (offsets[atoms] = edge count);
 *   ictc_neighbor_fill writes src [E], dst [E] (int64) and shift [E, 3].
 */
int64_t ictc_neighbor_workspace_bytes(int64_t atoms, const float* box, float cutoff);
int ictc_neighbor_count(const float* pos, int64_t atoms, const float* box, float cutoff, void* workspace,
                        int64_t workspace_bytes, int64_t* offsets, void* stream);
int ictc_neighbor_fill(const float* pos, int64_t atoms, const float* box, float cutoff, const void* workspace,
                       int64_t workspace_bytes, const int64_t* offsets, int64_t* src, int64_t* dst, float* shift,
                       void* stream);

/*
 * The same search with receivers restricted to atoms [0, receivers): neighbours
 * still range over all atoms.  Builds a rank's edges in a spatial decomposition,
 * where the local atoms are the owned ones followed by ghost copies and only
 * owned atoms receive messages (the owned-destination edge lists of
 * mace_ictc/interfaces/ascend_lammps.py:368-421).  offsets has receivers + 1
 * entries.
 */
int ictc_neighbor_count_receivers(const float* pos, int64_t atoms, int64_t receivers, const float* box,
                                  float cutoff, void* workspace, int64_t workspace_bytes, int64_t* offsets,
                                  void* stream);
int ictc_neighbor_fill_receivers(const float* pos, int64_t atoms, int64_t receivers, const float* box,
                                 float cutoff, const void* workspace, int64_t workspace_bytes,
                                 const int64_t* offsets, int64_t* src, int64_t* dst, float* shift, void* stream);

/*
 * Fused radial MLP of the MACE interaction (tcgen05 tensor cores, 3xTF32):
 *   gates = W4 s*silu(W3 s*silu(W2 s*silu(W1 f)))     (bias-free, s = 1.6791767923989418)
 * for edge embeddings f [E, F] (F <= 8), hidden width 64 and G gate columns
 * (a multiple of 64).  Replaces the radial network `fc` evaluated per edge in
 * mace_ictc/models/pure_cartesian_ictd_fix.py:1545-1553 (the gates of
 * radial_graph_message, ictc_o3/backends/ascend/capacity_message.py:109-179).
 *   ictc_radial_image_bytes: size of the packed weight image (-1 if unsupported).
 *   ictc_radial_pack: HOST function; packs w1 [64, F], w2 [64, 64], w3 [64, 64],
 *     w4 [G, 64] (row-major, nn.Linear [out, in]) into `image` (host memory) as
 *     TF32 hi/lo pairs in the kernels' shared-memory layout; copy it to the device.
 *   ictc_radial_forward: gates [E, G] from f [E, F].
 *   ictc_radial_backward: grad_f [E, F] from grad_gates [E, G]; grad_h3 [E, 64]
 *     is device scratch (dL/dh3).
 *   status: optional device int, set non-zero if a wait inside the kernel timed out.
 */
int64_t ictc_radial_image_bytes(int features, int hidden, int gates);
int ictc_radial_pack(const float* w1, const float* w2, const float* w3, const float* w4, int features, int hidden,
                     int gates, void* image, int64_t image_bytes);
int ictc_radial_forward(const void* image, const float* feats, float* gates, int64_t edges, int features,
                        int hidden, int gates_width, int* status, void* stream);
int ictc_radial_backward(const void* image, const float* feats, const float* grad_gates, float* grad_h3,
                         float* grad_feats, int64_t edges, int features, int hidden, int gates_width, int* status,
                         void* stream);

/*
 * Equivariant channel mixing of one degree block l (M = 2l+1) in the flat
 * [channel][M] feature layout, in place in the caller's rows:
 *   y[n*y_stride + y_offset + o*M + k] (+)= scale * sum_i W_s[o, i] x[n*x_stride + x_offset + i*M + k]
 * weight: [S, cout, cin]; s = tile_species[t] for the nodes of tile t.
 * tiles: [num_tiles, ictc_channel_mix_tile_nodes()] node ids (-1 padded), grouped
 * by species; NULL = contiguous tiles over all `nodes` with species 0.
 * accumulate: add into y instead of overwriting.  Replaces the per-degree linears
 * of mace_ictc/models/pure_cartesian_ictd_fix.py:335-392 (channel linears),
 * :629-661 (message_linear) and :2381-2440 (element-conditioned linears).
 */
int ictc_channel_mix_tile_nodes(void);
int ictc_channel_mix(const float* x, int64_t x_stride, int64_t x_offset, const float* weight, const int64_t* tiles,
                     const int32_t* tile_species, int64_t num_tiles, float* y, int64_t y_stride, int64_t y_offset,
                     int64_t nodes, int cin, int cout, int degree, float scale, int accumulate, void* stream);

/*
 * Self-test of the bounded waits used by the tensor-core kernels (no counterpart
 * in the reference).  One CTA waits on a shared-memory barrier; with arrive = 0
 * nothing arrives, so the wait must give up after limit_ns (<= 5 s) and the kernel
 * writes *status = 1 (device int) and returns; with arrive = 1 it writes 0.  The
 * CUDA context stays usable either way: this is how a lost handoff is reported.
 */
int ictc_wait_selftest(int* status, int64_t limit_ns, int arrive, void* stream);

/*
 * Allocation-free neighbour search.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory during a step (an MD engine
 * that owns all device buffers in its own pool, or a host program using this C
 * library without a CUDA-aware allocator to hand out scratch).
 * Same result as ictc_neighbor_count followed by ictc_neighbor_fill, but the
 * cell lists live in a fixed device array inside the library
 * (ictc_neighbor_noalloc_scratch_bytes() = 8 MiB, kept by every GPU that loads
 * the library until the process exits; about 650,000 atoms at liquid
 * densities).  Larger systems are rejected with ICTC_ERR_INVALID before any
 * work is queued.  The caller passes offsets [atoms + 1] and output buffers of
 * capacity max_edges; offsets[atoms] always receives the edge count, and the
 * edges are written only when that count is <= max_edges (read offsets[atoms]
 * after the stream completes to detect a too-small capacity).  Calls that
 * overlap on the GPU (other streams or threads) share the array and race;
 * serialise them.  Every call made outside stream capture looks up the array's
 * device address with that device current (so a context reset cannot leave a
 * stale address); a captured call reuses the last address looked up on its
 * device, so make a device's first call before any stream capture.  Nothing is
 * allocated or freed.
 */
int64_t ictc_neighbor_noalloc_scratch_bytes(void);
int ictc_neighbor_list_noalloc(const float* pos, int64_t atoms, const float* box, float cutoff, int64_t* offsets,
                               int64_t* src, int64_t* dst, float* shift, int64_t max_edges, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ICTC_CUDA_H */
