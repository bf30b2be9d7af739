"""Host-side choices of the dense projections (no GPU): how many token ranges a weight
gradient is split into when its output has too few tiles to fill the GPU."""
from spec_ep.ops.linear import wgrad_split


def test_wgrad_split_choice():
    assert wgrad_split(128, 2048, 4096, 148) == 16  # router: 8 tiles -> 128
    assert wgrad_split(5120, 2048, 4096, 148) == 1  # QKV fills the GPU
    assert wgrad_split(151936, 2048, 4096, 148) == 1  # LM head
    assert wgrad_split(128, 2048, 4160, 148) == 13  # 320-row ranges (multiples of 64)
    assert wgrad_split(128, 2048, 448, 148) == 1  # too few tokens to split


def test_wgrad_split_ranges_are_whole_64_row_steps():
    for T in range(512, 8193, 64):
        parts = wgrad_split(128, 2048, T, 148)
        assert T % parts == 0 and (T // parts) % 64 == 0 and T // parts >= 64
