"""Host layout of a packed prefill pass (hexgen2_b200.ops.varlen_table), on the CPU: the int32
table that hx_prefill_attention_varlen and hx_gemm_qkv_rotary_varlen read through pointers at
fixed offsets (row offsets at 0, slots at n + 1, start positions at 2n + 1, work items at the
returned index)."""
import pytest

from hexgen2_b200.ops import varlen_table


@pytest.mark.parametrize("lengths,slots", [([1], [0]), ([129, 1, 700, 128, 127, 300], [3, 0, 6, 1, 4, 2]),
                                           ([285, 750, 532, 1490], [7, 6, 5, 4]), ([128] * 5, list(range(5)))])
def test_varlen_table_layout(lengths, slots):
    values, n_items, items_at = varlen_table(lengths, slots)
    n = len(lengths)
    offs = values[:n + 1]
    assert offs[0] == 0 and all(offs[b + 1] - offs[b] == lengths[b] for b in range(n))
    assert values[n + 1:2 * n + 1] == slots
    assert values[2 * n + 1:3 * n + 1] == [0] * n  # prefill starts at position 0
    assert items_at % 2 == 0 and items_at in (3 * n + 1, 3 * n + 2)  # items are 8-byte int2
    items = [tuple(values[items_at + 2 * i:items_at + 2 * i + 2]) for i in range(n_items)]
    assert len(values) == items_at + 2 * n_items
    # Every (prompt, 128-query block) exactly once, the latest blocks (most causal work) first.
    want = {(b, q) for b, L in enumerate(lengths) for q in range(-(-L // 128))}
    assert set(items) == want and len(items) == len(want)
    assert [(-q, b) for b, q in items] == sorted((-q, b) for b, q in items)


@pytest.mark.parametrize("lengths,slots", [([], []), ([3, 4], [0]), ([3, 0], [0, 1]), ([5, -1], [0, 1])])
def test_varlen_table_rejects_bad_passes(lengths, slots):
    with pytest.raises(ValueError):
        varlen_table(lengths, slots)
