"""The decode split-length rule for rows of known length (used by the
tensor-parallel decoder): balanced splits of at most 64 blocks whose warp count
fits one wave, fills at least 40 % of its last wave, or makes three waves or
more on a 148-SM B200. The expected values are the best or within 1 % of the
best of a sweep on B200 (256 rows of 256 blocks, head_dim 128: one kv head 64,
two 52, four 52 (32 measured 0.7 % faster), eight 64)."""
import pytest

from serving_engine_b200.ops import decode_blocks_per_split


@pytest.mark.parametrize("hkv,expected", [(1, 64), (2, 52), (4, 52), (8, 64)])
def test_tp_shard_shapes(hkv, expected):
    # 256 sequences at 4096 tokens = 256 blocks per row (config 5 at TP = 8 / hkv)
    assert decode_blocks_per_split(256, hkv, 256, num_sms=148) == expected


def test_bounds():
    assert decode_blocks_per_split(1, 1, 4, num_sms=148) == 8       # rows shorter than a minimum split
    assert decode_blocks_per_split(4096, 8, 512, num_sms=148) == 64  # plenty of work: the longest split
    for items, hkv, blocks in [(64, 8, 512), (256, 1, 256), (37, 3, 100), (3, 1, 2000), (500, 2, 9)]:
        assert 8 <= decode_blocks_per_split(items, hkv, blocks, num_sms=148) <= 64


def test_chosen_split_count_makes_full_waves():
    slots = 148 * 12
    for items, hkv, blocks in [(64, 8, 512), (256, 1, 256), (256, 2, 256), (37, 3, 100), (128, 4, 300)]:
        bps = decode_blocks_per_split(items, hkv, blocks, num_sms=148)
        splits = -(-blocks // bps)
        assert bps == -(-blocks // splits)  # balanced: the row divided into equal parts
        waves = items * hkv * splits / slots
        assert waves <= 1.0 or waves >= 3.0 or waves - int(waves) >= 0.4 or bps == 8
