"""GGML tensor types and block geometry (the GGUF block table).

Parity: crates/hawking-core/src/gguf.rs:35-56 (GgmlType ids) and :87-111 (block_layout).
"""
from dataclasses import dataclass


class GgmlType:
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    I8 = 24
    I16 = 25
    I32 = 26
    I64 = 27
    F64 = 28
    BF16 = 30


@dataclass(frozen=True)
class BlockLayout:
    name: str
    block_elems: int
    block_bytes: int


LAYOUTS = {
    GgmlType.F32: BlockLayout("F32", 1, 4),
    GgmlType.F16: BlockLayout("F16", 1, 2),
    GgmlType.BF16: BlockLayout("BF16", 1, 2),
    GgmlType.F64: BlockLayout("F64", 1, 8),
    GgmlType.Q4_0: BlockLayout("Q4_0", 32, 18),
    GgmlType.Q4_1: BlockLayout("Q4_1", 32, 20),
    GgmlType.Q5_0: BlockLayout("Q5_0", 32, 22),
    GgmlType.Q5_1: BlockLayout("Q5_1", 32, 24),
    GgmlType.Q8_0: BlockLayout("Q8_0", 32, 34),
    GgmlType.Q8_1: BlockLayout("Q8_1", 32, 36),
    GgmlType.Q2_K: BlockLayout("Q2_K", 256, 84),
    GgmlType.Q3_K: BlockLayout("Q3_K", 256, 110),
    GgmlType.Q4_K: BlockLayout("Q4_K", 256, 144),
    GgmlType.Q5_K: BlockLayout("Q5_K", 256, 176),
    GgmlType.Q6_K: BlockLayout("Q6_K", 256, 210),
    GgmlType.Q8_K: BlockLayout("Q8_K", 256, 292),
    GgmlType.I8: BlockLayout("I8", 1, 1),
    GgmlType.I16: BlockLayout("I16", 1, 2),
    GgmlType.I32: BlockLayout("I32", 1, 4),
    GgmlType.I64: BlockLayout("I64", 1, 8),
}

BY_NAME = {v.name: k for k, v in LAYOUTS.items()}


def row_bytes(t: int, cols: int) -> int:
    lay = LAYOUTS[t]
    if cols % lay.block_elems:
        raise ValueError(f"{lay.name}: row length {cols} is not a multiple of {lay.block_elems}")
    return cols // lay.block_elems * lay.block_bytes


def type_id(t) -> int:
    if isinstance(t, str):
        return BY_NAME[t.upper()]
    return int(t)
