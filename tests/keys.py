"""numpy restatement of the vocab-parallel argmax keys (pyxis_b200/csrc/argmax.cu,
launch_argmax_keys / pick_keys_kernel), used to check the key scheme against the oracle's argmax
(src/output_head.rs:30-44) on the CPU, without a GPU."""
import numpy as np


def ordered(v: np.float32) -> int:
    """Order-preserving 32-bit image of a non-NaN float; -0.0 maps like +0.0."""
    if v == 0:
        v = np.float32(0.0)
    u = int(np.array([v], np.float32).view(np.uint32)[0])
    return (~u) & 0xFFFFFFFF if u & 0x80000000 else u | 0x80000000


def shard_key(v, lo: int) -> int:
    """One row's key for the shard v = values[lo:lo + len(v)] of a longer row."""
    v = np.asarray(v, np.float32)
    if lo == 0 and np.isnan(v[0]):
        return (1 << 64) - 1
    best = 0
    for i, x in enumerate(v):
        if np.isnan(x):
            continue
        k = (ordered(x) << 32) | (0xFFFFFFFF - (lo + i))
        best = max(best, k)
    return best


def pick(keys) -> int:
    m = max(int(k) for k in keys)
    return 0 if m == 0 else 0xFFFFFFFF - (m & 0xFFFFFFFF)


def element_key(x, g: int) -> int:
    """argmax_key_global (pyxis_b200/csrc/argmax.h): the key of one logit at global index g, as
    the tensor-core GEMV's epilogue builds it for every logit it writes."""
    x = np.float32(x)
    if np.isnan(x):
        return (1 << 64) - 1 if g == 0 else 0
    return (ordered(x) << 32) | (0xFFFFFFFF - g)


def epilogue_key(v, lo: int, rng) -> int:
    """The fused epilogue's key of a shard: element keys max-reduced in an arbitrary grouping and
    order (threads, warps, CTAs, then atomicMax into a slot that starts at 0)."""
    v = np.asarray(v, np.float32)
    keys = [element_key(x, lo + i) for i, x in enumerate(v)]
    order = rng.permutation(len(keys))
    slot = 0
    for chunk in np.array_split(order, max(1, int(rng.integers(1, 6)))):
        part = 0
        for i in chunk:
            part = max(part, keys[i])
        slot = max(slot, part)
    return slot
