"""Derived per-object state of the CUDA backend (device plans of a tensor product,
packed radial weights, symmetrised couplings, folded contraction tables, species
maps), kept on the object it belongs to.

That state is rebuilt on demand from the object's own parameters and buffers, and
it holds device handles (freed by their owners) and weak references, so it is left
out when the object is pickled or deep-copied: the copy starts with an empty cache
instead of sharing, or failing to serialise, the original's.
"""


class Transient:
    """A cache slot that pickles and deep-copies as empty."""

    __slots__ = ("value",)

    def __init__(self, value=None):
        self.value = value

    def __reduce__(self):
        return (Transient, ())

    def __deepcopy__(self, memo):
        return Transient()


def cache_of(obj, name: str) -> dict:
    """The cache dict ``name`` of ``obj``, created empty on first use (and after the
    object was unpickled or deep-copied)."""
    holder = obj.__dict__.get(name)
    if not isinstance(holder, Transient) or holder.value is None:
        holder = Transient({})
        obj.__dict__[name] = holder
    return holder.value
