"""The driver's smoke check (one small bucketed CAGRA build, bit-exact vs the oracle) as a GPU test."""
import pytest


@pytest.mark.gpu
def test_graft_entry_smoke():
    import __graft_entry__

    __graft_entry__.smoke()
