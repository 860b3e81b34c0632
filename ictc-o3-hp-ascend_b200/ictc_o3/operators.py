"""Public ICTC-O3 operators on the B200 CUDA backend.

Same names, arguments, layouts and error behaviour as the reference's public
API (``ictc_o3/operators.py``); the device is CUDA instead of an Ascend NPU and
every operator runs through libictc_cuda.so.  There is no host fallback.
"""
import torch
import torch.nn.functional as F

from ictc_o3.backends.cuda.linear import channel_linear, species_channel_linear
from ictc_o3.backends.cuda.runtime import require_cuda_fp32, strict_fp32


def _degree(value, name):
    if not isinstance(value, int) or isinstance(value, bool) or value < 0:
        raise ValueError(f"{name} must be a nonnegative integer")


def _positive_integer(value, name):
    if not isinstance(value, int) or isinstance(value, bool) or value < 1:
        raise ValueError(f"{name} must be a positive integer")


class EdgeTensorProduct(torch.nn.Module):
    """Path-preserving TP with live external gates (reference ``operators.py:19-138``).

    ir_mul stores each degree as [angular, channel]; mul_ir stores
    [channel, angular].  Output multiplicities keep the original path order.
    """

    def __init__(self, tp, *, input_lmax, edge_lmax, layout="ir_mul"):
        super().__init__()
        from ictc_o3.basis.ictd_irreps import EdgeWeightedPathPreservingTensorProduct
        if not isinstance(tp, EdgeWeightedPathPreservingTensorProduct):
            raise TypeError("Expected an ICTC path-preserving tensor product")
        _degree(input_lmax, "input_lmax")
        _degree(edge_lmax, "edge_lmax")
        require_cuda_fp32(tp.weight)
        if layout not in ("ir_mul", "mul_ir"):
            raise ValueError("layout must be ir_mul or mul_ir")
        if tp.internal_compute_dtype != torch.float32:
            raise ValueError("Tensor-product internal compute dtype must be FP32")
        if not tp.paths or any(i > input_lmax or j > edge_lmax for i, j, _ in tp.paths):
            raise ValueError("Declared input degrees must cover every tensor-product path")
        strict_fp32()
        self.tp, self.input_lmax, self.edge_lmax, self.layout = tp, input_lmax, edge_lmax, layout

    @classmethod
    def create(cls, *, channels=64, input_lmax=2, edge_lmax=2, output_lmax=None, layout="ir_mul",
               device="cuda"):
        _positive_integer(channels, "channels")
        _degree(input_lmax, "input_lmax")
        _degree(edge_lmax, "edge_lmax")
        output_lmax = input_lmax if output_lmax is None else output_lmax
        _degree(output_lmax, "output_lmax")
        if torch.device(device).type != "cuda":
            raise ValueError("This operator factory requires a CUDA device")
        from ictc_o3.basis.ictd_irreps import EdgeWeightedPathPreservingTensorProduct, operator_paths
        tp = EdgeWeightedPathPreservingTensorProduct(
            channels=channels, lmax=max(input_lmax, edge_lmax, output_lmax),
            allowed_paths=operator_paths(input_lmax, edge_lmax, output_lmax),
            internal_compute_dtype=torch.float32,
        ).to(device=device, dtype=torch.float32)
        with torch.no_grad():
            tp.weight.fill_(1.)
        tp.weight.requires_grad_(False)
        return cls(tp, input_lmax=input_lmax, edge_lmax=edge_lmax, layout=layout)

    @property
    def paths(self):
        return tuple(tuple(p) for p in self.tp.paths)

    @property
    def gate_width(self):
        return self.tp.num_paths * self.tp.channels

    @property
    def output_width(self):
        return sum(count * self.tp.channels * (2 * l + 1) for l, count in self.tp.path_counts_by_l.items())

    def pack_input(self, blocks):
        parts = []
        for l in range(self.input_lmax + 1):
            value = blocks[l]
            if value.shape[1:] != (self.tp.channels, 2 * l + 1):
                raise ValueError("Input block must have shape [E,C,2*l+1]")
            if self.layout == "ir_mul":
                value = value.transpose(1, 2)
            parts.append(value.reshape(value.shape[0], self.tp.channels * (2 * l + 1)))
        return torch.cat(parts, -1)

    def _check_packed(self, features, harmonics, rows):
        require_cuda_fp32(features, self.tp.weight)
        if features.ndim != 2 or features.shape[1] != self.tp.channels * (self.input_lmax + 1) ** 2:
            raise ValueError("Packed features must have shape [E,C*(L_in+1)^2]")
        require_cuda_fp32(harmonics, self.tp.weight)
        if harmonics.shape != (rows, (self.edge_lmax + 1) ** 2):
            raise ValueError("Harmonics must have shape [E,(L_edge+1)^2]")

    def unpack_output(self, output):
        result, offset = {}, 0
        for l in range(self.tp.lmax + 1):
            count, width = self.tp.path_counts_by_l.get(l, 0), 2 * l + 1
            span = count * self.tp.channels * width
            value = output[:, offset:offset + span]
            if self.layout == "ir_mul":
                value = value.reshape(output.shape[0], count, width, self.tp.channels).transpose(2, 3)
            result[l] = value.reshape(output.shape[0], count * self.tp.channels, width)
            offset += span
        return result

    def forward(self, features, harmonics, gates):
        from ictc_o3.backends.cuda.tensor_product import packed_product
        rows = features.shape[0]
        self._check_packed(features, harmonics, rows)
        if gates is not None:
            require_cuda_fp32(gates)
            if gates.shape not in ((rows, self.gate_width), (rows, self.tp.num_paths, self.tp.channels)):
                raise ValueError("External gates must have shape [E,P*C] or [E,P,C]")
        return packed_product(self.tp, self.layout, features, harmonics, gates)


class PackedGraphMessage(EdgeTensorProduct):
    """Packed node gather, CUDA TP and destination aggregation (reference ``operators.py:141-163``)."""

    def __init__(self, *args, edge_chunk_size=16384, **kwargs):
        super().__init__(*args, **kwargs)
        _positive_integer(edge_chunk_size, "edge_chunk_size")
        self.edge_chunk_size = edge_chunk_size

    @classmethod
    def create(cls, *, edge_chunk_size=16384, **kwargs):
        op = EdgeTensorProduct.create(**kwargs)
        return cls(op.tp, input_lmax=op.input_lmax, edge_lmax=op.edge_lmax,
                   layout=op.layout, edge_chunk_size=edge_chunk_size)

    def forward(self, features, harmonics, gates, src, dst, mask=None):
        for value in (src, dst):
            if value.ndim != 1 or value.dtype != torch.int64 or value.device != features.device:
                raise ValueError("Graph indices must be int64 vectors on the CUDA device")
        if dst.shape != src.shape:
            raise ValueError("Source and destination index shapes must match")
        require_cuda_fp32(features, self.tp.weight)
        if features.ndim != 2 or features.shape[1] != self.tp.channels * (self.input_lmax + 1) ** 2:
            raise ValueError("Packed features must have shape [E,C*(L_in+1)^2]")
        if harmonics.shape != (src.numel(), (self.edge_lmax + 1) ** 2):
            raise ValueError("Harmonics must have shape [E,(L_edge+1)^2]")
        require_cuda_fp32(harmonics, gates)
        from ictc_o3.backends.cuda.message import packed_graph_message
        return packed_graph_message(self.tp, self.layout, features, harmonics, gates, src, dst, mask)


class GraphMessage(PackedGraphMessage):
    """Dictionary block interface for the same graph message map."""

    def forward(self, features, harmonics, gates, src, dst, mask=None):
        from ictc_o3.backends.cuda.message import graph_message
        return graph_message(self.tp, features, harmonics, gates, src, dst, mask,
                             edge_chunk_size=self.edge_chunk_size)


def direction_harmonics(directions, lmax, *, policy="auto"):
    """Y_l(n) for l <= lmax as a list of [..., 2l+1] (reference ``operators.py:173-186``).

    Every policy evaluates the CUDA kernel; "reference" is accepted for API
    compatibility and selects the same kernel.
    """
    _degree(lmax, "lmax")
    if policy not in ("auto", "generated", "reference"):
        raise ValueError("policy must be auto, generated or reference")
    require_cuda_fp32(directions)
    from ictc_o3.basis.ictd_irreps import direction_harmonics_all
    return direction_harmonics_all(directions, lmax)


def configure_symmetric_contraction(module, *, policy="auto", training=False):
    """Select the CUDA contraction for a module (reference ``operators.py:189-201``).

    Accepts the bridge-U module the reference requires and the pure-ICTC one; both
    run on the same kernels."""
    from ictc_o3.ops.symmetric_contraction import (ICTDBridgeUSymmetricContractionSO3,
                                                   ICTDPureUSymmetricContractionSO3)
    if not isinstance(module, (ICTDBridgeUSymmetricContractionSO3, ICTDPureUSymmetricContractionSO3)):
        raise TypeError("Expected an ICTC bridge-U (or pure-ICTC) symmetric contraction")
    if policy not in ("auto", "generated", "reference"):
        raise ValueError("policy must be auto, generated or reference")
    require_cuda_fp32(*module.parameters())
    if module.correlation not in (1, 2, 3):
        raise ValueError("CUDA symmetric contraction supports correlation 1, 2 and 3")
    strict_fp32()
    module._cuda_hp = True
    return {"backend": "cuda", "selected": "generated"}


def create_symmetric_contraction(*, num_elements, lmax, target_lmax=None, channels=64,
                                 correlation=3, device="cuda", policy="generated", training=False):
    """Reference ``operators.py:204-218``, CUDA device: a bridge-U module (the
    reference's class), whose couplings are the ICTC ones until a reference state
    dict is loaded into it."""
    for value, name in ((num_elements, "num_elements"), (channels, "channels"), (correlation, "correlation")):
        _positive_integer(value, name)
    if correlation not in (1, 2, 3):
        raise ValueError("CUDA symmetric contraction supports correlation 1, 2 and 3")
    _degree(lmax, "lmax")
    target_lmax = lmax if target_lmax is None else target_lmax
    _degree(target_lmax, "target_lmax")
    if torch.device(device).type != "cuda":
        raise ValueError("This operator factory requires a CUDA device")
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3
    module = ICTDBridgeUSymmetricContractionSO3(num_elements=num_elements, channels=channels, lmax=lmax,
                                                target_lmax=target_lmax, correlation=correlation)
    module = module.to(device=device, dtype=torch.float32)
    configure_symmetric_contraction(module, policy=policy, training=training)
    return module


def normalized_silu(features, scale=1.):
    require_cuda_fp32(features)
    if not isinstance(scale, (int, float)) or isinstance(scale, bool):
        raise TypeError("scale must be a fixed numeric scalar")
    return F.silu(features) * float(scale)


__all__ = ["EdgeTensorProduct", "PackedGraphMessage", "GraphMessage", "direction_harmonics",
           "create_symmetric_contraction", "configure_symmetric_contraction",
           "channel_linear", "species_channel_linear", "normalized_silu", "strict_fp32"]
