"""Host-side rules of ``PagedModel``'s captured decode steps (no GPU needed)."""

from pager_hf.paged_model import _DecodeGraph


def test_graph_table_width_covers_blocks_and_tail_in_fixed_steps():
    """A captured step's block table holds the blocks plus the tail column, rounded up to a multiple
    of ``WIDTH_STEP``: a session re-captures once per ``WIDTH_STEP`` new blocks, not per block."""
    step = _DecodeGraph.WIDTH_STEP
    widths = [_DecodeGraph.width_for(nb) for nb in range(0, 5 * step)]
    for nb, w in enumerate(widths):
        assert w >= nb + 1 and w % step == 0 and w - (nb + 1) < step
    assert len(set(widths)) == 5  # one width per WIDTH_STEP blocks
