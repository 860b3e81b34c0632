from .adjoint_requirements import required_gradients

__all__ = ["required_gradients"]
