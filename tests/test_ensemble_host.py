"""ModelEnsemble host logic (no GPU): validation, weight totals, the one-hot
specialist rule and segment handling, as unblend/apply.py:63-219 and 730-760."""

from __future__ import annotations

import math

import pytest

from unblend_b200.apply import ModelEnsemble, ValidationError, _shift_plan


class _Stub:
    def __init__(self, sources=("drums", "bass", "other", "vocals"), sr=44100, ch=2, seg=7.8, norm=True):
        self.sources = list(sources)
        self.samplerate = sr
        self.audio_channels = ch
        self.max_allowed_segment = seg
        self.external_normalization = norm


def test_weights_and_totals():
    ens = ModelEnsemble([_Stub(), _Stub()], weights=[[1, 0.5, 0, 2], [0, 0.5, 1, 1]])
    assert ens.validated_weight_totals() == [1.0, 1.0, 1.0, 3.0]
    assert ModelEnsemble([_Stub(), _Stub(), _Stub()]).validated_weight_totals() == [3.0] * 4


@pytest.mark.parametrize("models,weights", [
    ([], None),
    ([_Stub(), _Stub(sources=("a", "b", "c", "d"))], None),
    ([_Stub(), _Stub(sr=48000)], None),
    ([_Stub(), _Stub(ch=1)], None),
    ([_Stub(), _Stub(norm=False)], None),
    ([_Stub(), _Stub(seg=math.inf)], None),
    ([_Stub(), _Stub()], [[1, 1, 1, 1]]),
    ([_Stub(), _Stub()], [[1, 1, 1], [1, 1, 1, 1]]),
    ([_Stub(), _Stub()], [[1, 1, 1, math.nan], [1, 1, 1, 1]]),
    ([_Stub(), _Stub()], [[1, 1, True, 1], [1, 1, 1, 1]]),
    ([_Stub(), _Stub()], [[1, 1, 1, 1], [-1, 0, 0, 0]]),  # zero total for "drums"
])
def test_invalid_ensembles_are_rejected(models, weights):
    with pytest.raises(ValidationError):
        ModelEnsemble(models, weights=weights)


def test_specialist_rule_and_segment():
    a, b = _Stub(seg=7.8), _Stub(seg=6.0)
    ens = ModelEnsemble([a, b], weights=[[1, 0, 0, 0], [0, 1, 1, 1]], segment=7.0)
    assert ens.specialist_for("drums") == 0
    assert ens.specialist_for("bass") is None  # row 1 is not one-hot
    assert ens.specialist_for("kazoo") is None and ens.specialist_for(None) is None
    assert a.max_allowed_segment == 7.0 and b.max_allowed_segment == 6.0
    assert ens.max_allowed_segment == 6.0
    with pytest.raises(NotImplementedError):
        ens(None)
    ft = ModelEnsemble([_Stub() for _ in range(4)], weights=[[float(i == j) for j in range(4)] for i in range(4)])
    assert [ft.specialist_for(s) for s in ft.sources] == [0, 1, 2, 3]


def test_shift_plan_is_round_major():
    import random

    random.seed(3)
    plan = _shift_plan(2, 3, 100, None)
    random.seed(3)
    draws = [random.randint(0, 100) for _ in range(6)]
    assert plan == [[draws[0], draws[3]], [draws[1], draws[4]], [draws[2], draws[5]]]
    assert _shift_plan(2, 2, 100, [4, 5]) == [[4, 5], [4, 5]]
    assert _shift_plan(0, 2, 100, None) == [[], []]
