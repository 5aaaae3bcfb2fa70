"""Drop-in contract with the reference's own engine (CPU; needs a reference checkout).

The reference's ``apply_model`` (unblend/apply.py:500-564) and
``Separator(model=...)`` (unblend/api.py:848-849) drive a module instance
through the ``SeparationModel`` contract (unblend/backends.py:36-59): device
moves, ``eval()``, ``parameters()``, ``sources``, ``samplerate``,
``audio_channels``, ``max_allowed_segment``, ``_fixed_batch_shape`` and
``model(batch)``. Here an :class:`HTDemucsCuda` instance goes through both
entry points with its attribute reads recorded; only its arithmetic is
replaced by the reference module's CPU forward (this machine has no GPU; the
GPU tests pin the CUDA forward to the reference's outputs). Every attribute the
engine reads must resolve on the instance itself, and the separations must
equal those of the reference module driven the same way.
"""

from __future__ import annotations

import sys

import pytest
import torch

from conftest import GOLDEN, reference_path
from unblend_b200.htdemucs import HTDemucsCuda
from unblend_b200.synth import htdemucs_config, htdemucs_state_dict, synth_track

REF = reference_path()
pytestmark = pytest.mark.skipif(REF is None, reason="reference checkout not found (set UNBLEND_REFERENCE)")
SMALL = dict(channels=8, bottom_channels=32, t_heads=4, t_layers=3, segment=0.5)


def _models():
    sys.path.insert(0, GOLDEN)
    from make_golden import import_reference

    unblend = import_reference(REF)
    import unblend.api  # noqa: F401

    cfg = htdemucs_config("htdemucs", **SMALL)
    torch.manual_seed(0)
    ref = unblend.htdemucs.HTDemucs(**{k: v for k, v in cfg.items() if k != "samplerate"},
                                    samplerate=cfg["samplerate"]).eval()
    reads: list[str] = []

    class Recorded(HTDemucsCuda):
        def __getattribute__(self, name):
            reads.append(name)
            return super().__getattribute__(name)

    fast = Recorded(cfg, ref.state_dict())
    seg = fast.segment_length

    def forward(mix: torch.Tensor) -> torch.Tensor:
        # The contract HTDemucsCuda.forward keeps: [B, C, T <= segment] -> [B, S, C, T].
        assert mix.dim() == 3 and mix.shape[-1] <= seg
        return ref(mix)

    object.__setattr__(fast, "forward", forward)
    return unblend, ref, fast, reads


def _own_attributes(m: HTDemucsCuda) -> set[str]:
    names = set(dir(type(m))) | set(vars(m))
    return names | set(m._modules) | set(m._parameters) | set(m._buffers)


def test_reference_apply_model_drives_the_cuda_model():
    unblend, ref, fast, reads = _models()
    mix = synth_track(1.6, 5)[None]
    with torch.no_grad():
        want = unblend.apply.apply_model(ref, mix, device="cpu", overlap=0.25, chunk_batch_size=2)
        reads.clear()
        got = unblend.apply.apply_model(fast, mix, device="cpu", overlap=0.25, chunk_batch_size=2)
    assert torch.equal(got, want)
    assert {"sources", "samplerate", "max_allowed_segment"} <= set(reads)
    assert set(reads) <= _own_attributes(fast) | {"forward"}


def test_reference_separator_accepts_the_cuda_model_instance():
    unblend, ref, fast, reads = _models()
    mix = synth_track(1.2, 6)
    # One shift round (the Separator's minimum) from the same seed on both sides.
    want = unblend.api.Separator(model=ref, device="cpu", chunk_batch_size=2).separate((mix, 44100), shifts=1,
                                                                                        seed=3)
    reads.clear()
    sep = unblend.api.Separator(model=fast, device="cpu", chunk_batch_size=2)
    got = sep.separate((mix, 44100), shifts=1, seed=3)
    assert sep.model is fast
    assert list(got.sources) == list(want.sources) == fast.sources
    for name in fast.sources:
        assert torch.equal(got.sources[name], want.sources[name])
    assert {"audio_channels", "samplerate", "sources"} <= set(reads)
    assert set(reads) <= _own_attributes(fast) | {"forward"}
