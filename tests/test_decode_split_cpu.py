"""The decode split-length rule for rows of known length (used by the
tensor-parallel decoder): the longest split of at most 32 blocks that still
gives about 1.5 waves of warps on a 148-SM B200. The expected values are the
ones a sweep on B200 found best (one kv head per rank at TP=8: 24-25 blocks;
two kv heads at TP=4 and more: 32)."""
import pytest

from serving_engine_b200.ops import decode_blocks_per_split


@pytest.mark.parametrize("hkv,expected", [(1, 25), (2, 32), (4, 32), (8, 32)])
def test_tp_shard_shapes(hkv, expected):
    # 256 sequences at 4096 tokens = 256 blocks per row (config 5 at TP = 8 / hkv)
    assert decode_blocks_per_split(256, hkv, 256, num_sms=148) == expected


def test_never_below_eight_or_above_thirtytwo():
    assert decode_blocks_per_split(1, 1, 4, num_sms=148) == 8      # too little work for 1.5 waves at any split
    assert decode_blocks_per_split(4096, 8, 512, num_sms=148) == 32


def test_enough_warps_at_the_chosen_split():
    for items, hkv, blocks in [(64, 8, 512), (256, 1, 256), (37, 3, 100)]:
        bps = decode_blocks_per_split(items, hkv, blocks, num_sms=148)
        warps = items * hkv * -(-blocks // bps)
        if bps > 8:
            assert warps >= 1.5 * 148 * 12
            assert items * hkv * -(-blocks // (bps + 1)) < 1.5 * 148 * 12 or bps == 32
