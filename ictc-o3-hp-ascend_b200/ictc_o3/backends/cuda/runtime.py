"""Runtime policy of the CUDA backend: eager FP32 on CUDA devices only.

Mirrors ``require_npu_fp32`` / ``strict_fp32`` of the reference
(``ictc_o3/backends/ascend/runtime.py:94-110``): precision is never changed
automatically, and matmuls run in full FP32 (TF32 off).
"""
import torch


def require_cuda_fp32(*values):
    if not values or any(v.device.type != "cuda" or v.dtype != torch.float32 for v in values):
        raise ValueError("The CUDA backend requires CUDA FP32 tensors; precision is never changed automatically")
    if any(v.device != values[0].device for v in values):
        raise ValueError("All operands must be on the same CUDA device")
    if torch.is_autocast_enabled("cuda"):
        raise ValueError("The CUDA backend requires autocast to be disabled")
    if torch.compiler.is_compiling() or torch._C._are_functorch_transforms_active():
        raise ValueError("The CUDA backend requires ordinary eager autograd")


def strict_fp32():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
