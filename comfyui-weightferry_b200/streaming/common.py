"""Flat block layouts (streaming/common.py of the reference, :87-120): every streamed block's parameters live in one
flat buffer, each at a 256-byte aligned offset, so that one copy moves a whole block and views bind its params."""

_ALIGN = 256  # bytes between parameter starts in a flat buffer


def _nbytes(shape, itemsize):
    n = 1
    for d in shape:
        n *= int(d)
    return n * int(itemsize)


def flat_layout(sizes):
    """Byte offsets of consecutive items of the given byte sizes in one flat buffer (each aligned to _ALIGN), and the
    total size (aligned)."""
    offsets, off = [], 0
    for sz in sizes:
        off = (off + _ALIGN - 1) // _ALIGN * _ALIGN
        offsets.append(off)
        off += int(sz)
    return offsets, (off + _ALIGN - 1) // _ALIGN * _ALIGN


def views(flat, sizes, offsets):
    """uint8 views of the items in a flat uint8 tensor."""
    return [flat[o:o + int(sz)] for sz, o in zip(sizes, offsets)]
