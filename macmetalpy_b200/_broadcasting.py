"""NumPy broadcasting rules (mirrors ``src/macmetalpy/_broadcasting.py:8-76``).

Unlike the reference, broadcast operands are never materialised
(``ndarray._gpu_broadcast_to``, ``ndarray.py:515-545``): a broadcast
dimension becomes a stride-0 dimension that the fused kernel indexes
directly.
"""

from __future__ import annotations

__all__ = ["broadcast_shapes", "broadcast_strides", "needs_broadcast"]


def broadcast_shapes(*shapes: tuple) -> tuple:
    """Broadcast shape of ``shapes``; ``ValueError`` if incompatible."""
    if not shapes:
        return ()
    first = None
    for s in shapes:  # fast path: every non-scalar shape equal
        if s:
            if first is None:
                first = s
            elif s != first:
                break
    else:
        return tuple(first) if first is not None else ()
    ndim = max(len(s) for s in shapes)
    out = []
    for axis in range(-ndim, 0):
        dims = [s[axis] if len(s) >= -axis else 1 for s in shapes]
        non_one = {d for d in dims if d != 1}
        if len(non_one) > 1:
            raise ValueError(f"Shape mismatch: cannot broadcast shapes {shapes}")
        out.append(non_one.pop() if non_one else 1)
    return tuple(out)


def broadcast_strides(shape: tuple, target_shape: tuple, strides: tuple) -> tuple:
    """Element strides of ``shape``/``strides`` viewed as ``target_shape``.

    Stretched (size 1 -> n) and prepended dimensions get stride 0.
    """
    nd = len(target_shape) - len(shape)
    if nd < 0:
        raise ValueError(f"Cannot broadcast {shape} to {target_shape}")
    out = [0] * nd
    for size, tsize, st in zip(shape, target_shape[nd:], strides):
        if size == tsize:
            out.append(st if size != 1 else 0)
        elif size == 1:
            out.append(0)
        else:
            raise ValueError(f"Cannot broadcast dimension {size} to {tsize}")
    return tuple(out)


def needs_broadcast(shape1: tuple, shape2: tuple) -> bool:
    """True if the two shapes differ (so broadcasting is needed)."""
    return tuple(shape1) != tuple(shape2)
