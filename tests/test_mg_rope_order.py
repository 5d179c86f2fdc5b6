"""RoPE-pair packing order of QKV matrices (ops/mg.py rope_pair_rows): a permutation of the rows
in which packed tile rows r and r + 8 of every 16-row group of a q / k head are the two members of
one rotation pair, for both RoPE styles and partial rotation; v rows keep their order."""
import pytest

torch = pytest.importorskip("torch")

from hawking_b200.ops.mg import rope_pair_rows  # noqa: E402


@pytest.mark.parametrize("hd,rot,style", [(64, 64, 0), (64, 64, 1), (128, 128, 0), (128, 128, 1), (128, 64, 1),
                                          (128, 32, 0), (64, 16, 1)])
def test_rope_pair_rows(hd, rot, style):
    heads, n = 5, 7 * hd  # 5 q + k heads, then 2 v heads
    p = rope_pair_rows(heads, hd, rot, style, n)
    assert sorted(p.tolist()) == list(range(n))
    assert p[heads * hd:].tolist() == list(range(heads * hd, n))
    for R in range(0, heads * hd, 16):
        for r in range(8):
            a, b = int(p[R + r]), int(p[R + r + 8])
            assert a // hd == b // hd == R // hd
            a, b = a % hd, b % hd
            if a < rot:
                if style == 0:
                    assert a % 2 == 0 and b == a + 1
                else:
                    assert a < rot // 2 and b == a + rot // 2
            else:
                assert b >= rot


def test_rope_pair_rows_rejects_unaligned():
    with pytest.raises(ValueError):
        rope_pair_rows(2, 72, 72, 0, 144)
