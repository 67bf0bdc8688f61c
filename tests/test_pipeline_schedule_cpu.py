"""1F1B pipeline schedule and message tags (pure host logic).

Behaviour follows the reference's tests/test_runtime_pipeline.py: stable tags per micro-batch, warm-up of
min(pp - rank - 1, M) forwards, then one forward / one backward, then the remaining backwards."""
from types import SimpleNamespace

import pytest

from nano_train_b200.parallel.pipeline import activation_tag, execute_1f1b_schedule, grad_tag, label_tag


def test_tags_are_stable_and_disjoint():
    assert (activation_tag(0), grad_tag(0), label_tag(0)) == (10_000, 20_000, 30_000)
    assert (activation_tag(7), grad_tag(7), label_tag(7)) == (10_007, 20_007, 30_007)
    tags = [f(mb) for f in (activation_tag, grad_tag, label_tag) for mb in range(512)]
    assert len(set(tags)) == len(tags)


def _order(pp, rank, m):
    ev = []
    execute_1f1b_schedule(SimpleNamespace(pipeline_model_parallel_size=pp, pipeline_model_parallel_rank=rank), m,
                          run_forward=lambda i: ev.append(("F", i)), run_backward=lambda i: ev.append(("B", i)))
    return ev


def test_1f1b_order_for_a_four_stage_pipeline():
    assert _order(4, 0, 6) == [("F", 0), ("F", 1), ("F", 2), ("F", 3), ("B", 0), ("F", 4), ("B", 1), ("F", 5),
                               ("B", 2), ("B", 3), ("B", 4), ("B", 5)]
    assert _order(4, 3, 3) == [("F", 0), ("B", 0), ("F", 1), ("B", 1), ("F", 2), ("B", 2)]
    # fewer micro-batches than warm-up slots: all forwards, then all backwards
    assert _order(4, 0, 2) == [("F", 0), ("F", 1), ("B", 0), ("B", 1)]


@pytest.mark.parametrize("pp", [2, 3, 4, 8])
@pytest.mark.parametrize("m", [1, 2, 5, 8, 13])
def test_1f1b_invariants(pp, m):
    for rank in range(pp):
        ev = _order(pp, rank, m)
        assert sorted(i for k, i in ev if k == "F") == list(range(m))
        assert [i for k, i in ev if k == "B"] == list(range(m))  # backwards in micro-batch order
        in_flight, peak = 0, 0
        for k, i in ev:
            if k == "B":
                assert ("F", i) in ev[:ev.index(("B", i))]
            in_flight += 1 if k == "F" else -1
            peak = max(peak, in_flight)
        # activations held at once: warm-up depth + 1, which is what bounds 1F1B's memory
        assert peak == min(pp - rank, m)
