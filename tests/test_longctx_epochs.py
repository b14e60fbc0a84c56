"""Host side of the peer exchange's epochs (no GPU): the staged base wraps like a u32 and
the kernels' wrap-safe comparison keeps waiting for a flag one epoch behind."""

import pytest

from shellsmith_b200.longctx import epoch_base


def _u32(x: int) -> int:
    return x & 0xFFFFFFFF


def _reached(flag: int, want: int) -> bool:
    """The device test (int)(flag - want) >= 0 on 32-bit words."""
    d = _u32(flag - want)
    return (d - (1 << 32) if d >= 1 << 31 else d) >= 0


@pytest.mark.parametrize("layers", [2, 12])
@pytest.mark.parametrize("token", [0, 1, (1 << 31) // 12, (1 << 31) // 12 + 1,
                                   (1 << 32) // 12 - 1, (1 << 32) // 12 + 5, 10 ** 9])
def test_epochs_wrap_and_compare(token, layers):
    base = epoch_base(token, layers)
    assert -(1 << 31) <= base < (1 << 31)
    assert _u32(base) == _u32(token * layers)
    for layer in range(layers):
        want = _u32(base + layer + 1)
        assert _reached(want, want) and _reached(_u32(want + 1), want)
        assert not _reached(_u32(want - 1), want)
    # The next token's first epoch follows this token's last one.
    assert _u32(epoch_base(token + 1, layers) + 1) == _u32(base + layers + 1)
