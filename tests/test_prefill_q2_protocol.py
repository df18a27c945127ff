"""The synchronisation protocol of the two-query-tile prefill kernel (csrc/prefill_q2.cu),
checked without a GPU: an executable model of its roles, mbarriers and in-order tensor-core
execution (tests/q2_protocol_model.py) runs random work lists under random interleavings with no
deadlock, no aliased parity wait and no stale read, and each deliberate protocol mistake in the
model is reported."""
import pytest

import q2_protocol_model as model


def test_protocol_holds_on_random_work():
    assert model.check(trials=500, seed=1) is None


@pytest.mark.parametrize("mutation", model.MUTATIONS)
def test_model_reports_each_planted_mistake(mutation):
    assert model.check(trials=50, seed=2, mutation=mutation) is not None
