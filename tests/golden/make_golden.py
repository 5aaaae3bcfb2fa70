"""Generate the golden fixtures from the reference implementation itself.

Run from the repository root with a checkout of the reference project (the
path argument, else ``$UNBLEND_REFERENCE``, else ``reference`` beside this
repository)::

    python tests/golden/make_golden.py [<reference checkout> [configs|roformer|ensemble|melband|scnet]]

It imports the reference (``torchcodec`` is stubbed: the reference only uses it
for file decode/encode in unblend/api.py:20-21), builds each model exactly as
the registry does under ``torch.manual_seed(seed)`` (unblend/repo.py:121-143),
checks that ``unblend_b200.synth.htdemucs_state_dict`` reproduces those weights
bit for bit, and saves the reference's fp32 CPU outputs on synthetic audio:

* ``htdemucs_small.pt``   reduced-width HTDemucs (0.5 s segment), batch 2,
  full outputs of ``HTDemucs.forward`` (unblend/htdemucs.py:650).
* ``htdemucs_full.pt``    registry ``htdemucs`` (4 stems) on a 1 s clip, every
  5th output sample plus per-stem sums / sums of squares of the full output.
* ``htdemucs_6s_full.pt`` registry ``htdemucs_6s`` (seed 2), same summaries.
* ``apply_small.pt``      ``apply_model`` (unblend/apply.py:500) with the
  reduced model over a 4-segment track, shifts 0 and shifts 1 (offsets drawn
  after ``random.seed(5)``), every 7th output sample plus full sums.
* ``bsroformer_small.pt`` reduced BS-RoFormer (dim 64, depth 2, 4 heads of 16,
  seed 3), batch 2 on 0.5 s, full outputs of ``BSRoformer.forward``
  (unblend/roformer.py:1312).
* ``bsroformer_full.pt``  the measured BS-RoFormer (dim 512, depth 12, seed 3)
  on a 1 s clip, every 5th output sample plus per-stem sums.
* ``bsroformer_apply.pt`` ``apply_model`` with the reduced BS-RoFormer set up by
  ``configure_inference`` for 0.5 s segments and a complement stem
  (sources ["vocals", "other"]), over a 4-segment track.
* ``ensemble_small.pt``  ``apply_model`` on a ``ModelEnsemble`` of two reduced
  HTDemucs models (seeds 0 and 7): per-source weights with one shift round, and
  one-hot rows with ``use_only_stem`` ("drums" takes the specialist shortcut,
  "bass" does not), every 7th output sample plus full sums.
* ``melband_small.pt``   reduced Mel-Band RoFormer (dim 32, depth 2, 12 mel
  bands, seed 5), batch 2 on 0.5 s, full outputs of ``MelBandRoformer.forward``
  (unblend/roformer.py:1513), plus the band gather indices.
* ``melband_kim.pt``      the registry ``melband_roformer_kim`` configuration
  (dim 384, depth 6, 60 bands, seed 6) set up by ``configure_inference`` with a
  complement stem, on a 1 s clip: every 5th output sample plus per-stem sums.

``python tests/golden/make_golden.py <reference> configs`` writes the fixtures
of two measured configurations (their inputs are regenerated from the seed by
``synth_track``; ``mix_digest`` pins that):

* ``htdemucs_cfg0.pt``    the registry ``htdemucs`` (seed 0) through
  ``apply_model`` on a 10 s clip (seed 0), batch 1, shifts 0, overlap 0.25:
  every 16th output sample, full-resolution windows at the start, around both
  edges of the first chunk overlap and at the end, plus per-stem sums.
* ``htdemucs_6s_cfg2.pt`` the registry ``htdemucs_6s`` (seed 2) through
  ``apply_model`` with one shift round (offset drawn after ``random.seed(2)``)
  on a 16 s clip (seed 4), batch 4: the vocals stem (every 16th sample and the
  same windows) plus per-stem sums of all six stems.

``... scnet`` writes the SCNet fixtures (unblend/scnet.py):

* ``scnet_small_reduced.pt`` the masked architecture with reduced widths (dims
  4/16/32/32, two dual-path layers, seed 7), batch 2 on 0.5 s, full outputs.
* ``scnet_plain_reduced.pt`` the plain architecture with the xl band layout and
  reduced widths (seed 8), batch 2 on 0.5 s, full outputs.
* ``scnet_small_full.pt`` / ``scnet_xl_full.pt`` the registry ``scnet_small``
  (seed 9) and ``scnet_xl_wide_v5`` (seed 10) on a 1 s clip: every 5th output
  sample plus per-stem sums.
* ``scnet_apply.pt`` ``apply_model`` with the registry ``scnet_small`` over a
  16 s track (two 11 s segments), batch 2: every 16th sample, windows, sums.

The fixtures hold only outputs and small inputs; weights are regenerated from
the seed on the fly, and ``weights_digest`` pins that regeneration.
"""

from __future__ import annotations

import hashlib
import os
import random
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from unblend_b200.synth import (  # noqa: E402
    bsroformer_config,
    bsroformer_state_dict,
    melband_config,
    melband_state_dict,
    htdemucs_config,
    scnet_config,
    scnet_state_dict,
    htdemucs_state_dict,
    synth_track,
)

SMALL_OVERRIDES = dict(channels=8, bottom_channels=32, t_heads=4, t_layers=3, segment=0.5)
ROFORMER_SMALL = dict(dim=64, depth=2, heads=4, dim_head=16)


def reference_path() -> str:
    """The reference checkout: ``$UNBLEND_REFERENCE``, else ``reference`` beside this repository."""
    repo = os.path.dirname(os.path.dirname(HERE))
    path = os.environ.get("UNBLEND_REFERENCE") or os.path.join(os.path.dirname(repo), "reference")
    if not os.path.isdir(os.path.join(path, "unblend")):
        raise SystemExit(f"reference checkout not found at {path}; set UNBLEND_REFERENCE")
    return path


def import_reference(path: str):
    """Import the reference ``unblend`` package with ``torchcodec`` stubbed."""
    for name in ("torchcodec", "torchcodec.decoders", "torchcodec.encoders"):
        mod = types.ModuleType(name)
        mod.AudioDecoder = object
        mod.AudioEncoder = object
        sys.modules.setdefault(name, mod)
    if path not in sys.path:
        sys.path.insert(0, path)
    import unblend  # noqa: F401
    import unblend.apply
    import unblend.htdemucs
    return unblend


def weights_digest(sd: dict) -> str:
    """sha256 over every tensor's name and raw float32 bytes, in key order."""
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def _summary(y: torch.Tensor) -> dict:
    """Per-stem sum and sum of squares over a ``[B, S, C, L]`` output (float64)."""
    yd = y.double()
    return {"sum": yd.sum(dim=(0, 2, 3)), "sumsq": (yd * yd).sum(dim=(0, 2, 3))}


def build_reference(unblend, cfg: dict, seed: int):
    torch.manual_seed(seed)
    model = unblend.htdemucs.HTDemucs(**cfg).eval()
    mine = htdemucs_state_dict(cfg, seed)
    ref = model.state_dict()
    assert set(ref) == set(mine), "state_dict keys differ"
    for k in ref:
        assert torch.equal(ref[k], mine[k]), f"weight {k} differs"
    return model, weights_digest(mine)


def main(ref_path: str) -> None:
    unblend = import_reference(ref_path)
    torch.set_num_threads(os.cpu_count() or 1)
    with torch.inference_mode():
        # Reduced model, full outputs.
        cfg = htdemucs_config("htdemucs", **SMALL_OVERRIDES)
        model, digest = build_reference(unblend, cfg, 0)
        mix = torch.stack([synth_track(0.15, 10), synth_track(0.15, 11)])
        out = model(mix)
        torch.save({"config": cfg, "seed": 0, "weights_digest": digest, "mix": mix, "out": out.clone()},
                   os.path.join(HERE, "htdemucs_small.pt"))

        # apply_model over a 4-segment track with the reduced model.
        track = synth_track(1.3, 1)[None]
        res = {"config": cfg, "seed": 0, "weights_digest": digest, "mix": track,
               "overlap": 0.25, "chunk_batch_size": 3, "decimate": 7}
        y0 = unblend.apply.apply_model(model, track, device="cpu", shifts=0, overlap=0.25,
                                       chunk_batch_size=3)
        res["shifts0"] = {"out": y0[..., ::7].clone(), **_summary(y0)}
        random.seed(5)
        offsets = [random.randint(0, int(0.5 * cfg["samplerate"]))]
        random.seed(5)
        y1 = unblend.apply.apply_model(model, track, device="cpu", shifts=1, overlap=0.25,
                                       chunk_batch_size=3)
        res["shifts1"] = {"out": y1[..., ::7].clone(), "offsets": offsets, **_summary(y1)}
        torch.save(res, os.path.join(HERE, "apply_small.pt"))

        # Registry configurations on a 1 s clip (padded to the 7.8 s segment).
        for name, seed, fname in (("htdemucs", 0, "htdemucs_full.pt"),
                                  ("htdemucs_6s", 2, "htdemucs_6s_full.pt")):
            cfg = htdemucs_config(name)
            model, digest = build_reference(unblend, cfg, seed)
            mix = synth_track(1.0, 0)[None]
            out = model(mix)
            torch.save({"config": cfg, "seed": seed, "weights_digest": digest, "mix": mix,
                        "decimate": 5, "out": out[..., ::5].clone(), **_summary(out)},
                       os.path.join(HERE, fname))
    main_roformer(unblend)
    print("fixtures written to", HERE)


CFG_DECIMATE = 16
CFG_WINDOW = 2048


def config_windows(length: int, segment: int, stride: int) -> list[int]:
    """Starts of the full-resolution windows: the track start, both edges of the
    first chunk overlap, and the end."""
    return [0, stride - CFG_WINDOW // 2, segment - CFG_WINDOW // 2, length - CFG_WINDOW]


def _config_record(y: torch.Tensor, windows: list[int]) -> dict:
    """Decimated output, full-resolution windows and per-stem sums of ``y`` [1, S, C, L]."""
    return {"decimate": CFG_DECIMATE, "out": y[..., ::CFG_DECIMATE].clone(), "windows": windows,
            "window": CFG_WINDOW, "win_out": torch.stack([y[..., w:w + CFG_WINDOW] for w in windows]).clone(),
            **_summary(y)}


def mix_digest(x: torch.Tensor) -> str:
    return hashlib.sha256(x.contiguous().numpy().tobytes()).hexdigest()


def main_configs(unblend) -> None:
    """Fixtures of the 10 s registry clip (configs 0) and the 6-source vocals run with one shift round."""
    torch.set_num_threads(os.cpu_count() or 1)
    with torch.inference_mode():
        cfg = htdemucs_config("htdemucs")
        model, digest = build_reference(unblend, cfg, 0)
        mix = synth_track(10.0, 0)[None]
        y = unblend.apply.apply_model(model, mix, device="cpu", shifts=0, overlap=0.25, chunk_batch_size=1)
        seg = int(round(cfg["samplerate"] * cfg["segment"]))
        win = config_windows(mix.shape[-1], seg, int(0.75 * seg))
        torch.save({"config": cfg, "seed": 0, "weights_digest": digest, "mix_seconds": 10.0, "mix_seed": 0,
                    "mix_digest": mix_digest(mix), "overlap": 0.25, "chunk_batch_size": 1, "shifts": 0,
                    **_config_record(y, win)}, os.path.join(HERE, "htdemucs_cfg0.pt"))

        cfg = htdemucs_config("htdemucs_6s")
        model, digest = build_reference(unblend, cfg, 2)
        mix = synth_track(16.0, 4)[None]
        random.seed(2)
        offsets = [random.randint(0, int(0.5 * cfg["samplerate"]))]
        random.seed(2)
        y = unblend.apply.apply_model(model, mix, device="cpu", shifts=1, overlap=0.25, chunk_batch_size=4)
        v = cfg["sources"].index("vocals")
        rec = _config_record(y[:, v:v + 1], win)
        rec["stem_sum"], rec["stem_sumsq"] = _summary(y)["sum"], _summary(y)["sumsq"]
        torch.save({"config": cfg, "seed": 2, "weights_digest": digest, "mix_seconds": 16.0, "mix_seed": 4,
                    "mix_digest": mix_digest(mix), "overlap": 0.25, "chunk_batch_size": 4, "shifts": 1,
                    "offsets": offsets, "stem": "vocals", **rec}, os.path.join(HERE, "htdemucs_6s_cfg2.pt"))
    print("config fixtures written to", HERE)


def build_scnet(unblend, cfg: dict, seed: int):
    """``manual_seed(seed); build_scnet(...)``, checked against ``scnet_state_dict``."""
    import unblend.scnet

    torch.manual_seed(seed)
    kw = {k: v for k, v in cfg.items() if k not in ("architecture", "sources", "samplerate", "segment_samples")}
    model = unblend.scnet.build_scnet(cfg["architecture"], kw, sources=cfg["sources"], samplerate=cfg["samplerate"],
                                      segment_samples=cfg["segment_samples"])
    mine = scnet_state_dict(cfg, seed)
    ref = model.state_dict()
    assert set(ref) == set(mine), "state_dict keys differ"
    for k in ref:
        assert torch.equal(ref[k], mine[k]), f"weight {k} differs"
    return model, weights_digest(mine)


def main_scnet(unblend) -> None:
    """SCNet fixtures (reduced masked and plain models, registry configurations, apply_model)."""
    torch.set_num_threads(os.cpu_count() or 1)
    reduced = dict(dims=[4, 16, 32, 32], num_dplayer=2, conv_depths=[1, 1, 1])
    with torch.inference_mode():
        for name, seed, fname, over in (("scnet_small", 7, "scnet_small_reduced.pt", reduced),
                                        ("scnet_xl_wide_v5", 8, "scnet_plain_reduced.pt",
                                         dict(reduced, conv_depths=[2, 1, 1]))):
            cfg = scnet_config(name, **over)
            model, digest = build_scnet(unblend, cfg, seed)
            mix = torch.stack([synth_track(0.5, 40), synth_track(0.5, 41)])
            torch.save({"config": cfg, "seed": seed, "weights_digest": digest, "mix": mix,
                        "out": model(mix).clone()}, os.path.join(HERE, fname))
        for name, seed, fname in (("scnet_small", 9, "scnet_small_full.pt"), ("scnet_xl_wide_v5", 10, "scnet_xl_full.pt")):
            cfg = scnet_config(name)
            model, digest = build_scnet(unblend, cfg, seed)
            mix = synth_track(1.0, 42)[None]
            out = model(mix)
            torch.save({"config": cfg, "seed": seed, "weights_digest": digest, "mix": mix,
                        "decimate": 5, "out": out[..., ::5].clone(), **_summary(out)}, os.path.join(HERE, fname))
        cfg = scnet_config("scnet_small")
        model, digest = build_scnet(unblend, cfg, 9)
        mix = synth_track(16.0, 43)[None]
        y = unblend.apply.apply_model(model, mix, device="cpu", shifts=0, overlap=0.25, chunk_batch_size=2)
        seg = cfg["segment_samples"]
        win = config_windows(mix.shape[-1], seg, int(0.75 * seg))
        torch.save({"config": cfg, "seed": 9, "weights_digest": digest, "mix_seconds": 16.0, "mix_seed": 43,
                    "mix_digest": mix_digest(mix), "overlap": 0.25, "chunk_batch_size": 2, "shifts": 0,
                    **_config_record(y, win)}, os.path.join(HERE, "scnet_apply.pt"))
    print("SCNet fixtures written to", HERE)


def build_roformer(unblend, cfg: dict, seed: int):
    """``manual_seed(seed); BSRoformer(**cfg)``, checked against ``bsroformer_state_dict``."""
    import unblend.roformer

    torch.manual_seed(seed)
    model = unblend.roformer.BSRoformer(**cfg).eval()
    mine = bsroformer_state_dict(cfg, seed)
    ref = model.state_dict()
    assert set(ref) == set(mine), "state_dict keys differ"
    for k in ref:
        assert torch.equal(ref[k], mine[k]), f"weight {k} differs"
    return model, weights_digest(mine)


def main_roformer(unblend) -> None:
    """BS-RoFormer fixtures (reduced model, measured configuration, apply_model)."""
    with torch.inference_mode():
        cfg = bsroformer_config(**ROFORMER_SMALL)
        model, digest = build_roformer(unblend, cfg, 3)
        mix = torch.stack([synth_track(0.5, 20), synth_track(0.5, 21)])
        out = model(mix)
        torch.save({"config": cfg, "seed": 3, "weights_digest": digest, "mix": mix, "out": out.clone()},
                   os.path.join(HERE, "bsroformer_small.pt"))

        model.configure_inference(sources=["vocals", "other"], samplerate=44100, segment_samples=22050)
        track = synth_track(1.3, 22)[None]
        y = unblend.apply.apply_model(model, track, device="cpu", shifts=0, overlap=0.25, chunk_batch_size=3)
        torch.save({"config": cfg, "seed": 3, "weights_digest": digest, "mix": track, "segment_samples": 22050,
                    "sources": ["vocals", "other"], "overlap": 0.25, "chunk_batch_size": 3, "decimate": 7,
                    "out": y[..., ::7].clone(), **_summary(y)}, os.path.join(HERE, "bsroformer_apply.pt"))

        cfg = bsroformer_config()
        model, digest = build_roformer(unblend, cfg, 3)
        mix = synth_track(1.0, 23)[None]
        out = model(mix)
        torch.save({"config": cfg, "seed": 3, "weights_digest": digest, "mix": mix, "decimate": 5,
                    "out": out[..., ::5].clone(), **_summary(out)}, os.path.join(HERE, "bsroformer_full.pt"))


def main_ensemble(unblend) -> None:
    """ModelEnsemble fixtures: two reduced HTDemucs members (seeds 0 and 7) under apply_model."""
    torch.set_num_threads(os.cpu_count() or 1)
    with torch.inference_mode():
        cfg = htdemucs_config("htdemucs", **SMALL_OVERRIDES)
        m0, d0 = build_reference(unblend, cfg, 0)
        m7, d7 = build_reference(unblend, cfg, 7)
        track = synth_track(1.3, 3)[None]
        res = {"config": cfg, "seeds": [0, 7], "digests": [d0, d7], "mix": track, "overlap": 0.25,
               "chunk_batch_size": 3, "decimate": 7}
        weights = [[1.0, 0.5, 0.0, 2.0], [0.0, 0.5, 1.0, 1.0]]
        ens = unblend.apply.ModelEnsemble([m0, m7], weights=weights)
        random.seed(9)
        offsets = [random.randint(0, int(0.5 * cfg["samplerate"]))]
        random.seed(9)
        y = unblend.apply.apply_model(ens, track, device="cpu", shifts=1, overlap=0.25, chunk_batch_size=3)
        res["weighted"] = {"weights": weights, "offsets": offsets, "out": y[..., ::7].clone(), **_summary(y)}
        onehot = [[1.0, 0.0, 0.0, 0.0], [0.0, 1.0, 1.0, 1.0]]
        ens = unblend.apply.ModelEnsemble([m0, m7], weights=onehot)
        for stem in ("drums", "bass"):
            y = unblend.apply.apply_model(ens, track, device="cpu", shifts=0, overlap=0.25, chunk_batch_size=3,
                                          use_only_stem=stem)
            res[f"only_{stem}"] = {"weights": onehot, "out": y[..., ::7].clone(), **_summary(y)}
        torch.save(res, os.path.join(HERE, "ensemble_small.pt"))


MELBAND_SMALL = dict(dim=32, depth=2, num_bands=12, heads=2, dim_head=16, mask_estimator_depth=1)


def build_melband(unblend, cfg: dict, seed: int):
    """``manual_seed(seed); MelBandRoformer(**cfg)``, checked against ``melband_state_dict``."""
    import unblend.roformer

    torch.manual_seed(seed)
    model = unblend.roformer.MelBandRoformer(**cfg).eval()
    mine = melband_state_dict(cfg, seed)
    ref = model.state_dict()
    assert set(ref) == set(mine), "state_dict keys differ"
    for k in ref:
        assert torch.equal(ref[k], mine[k]), f"weight {k} differs"
    return model, weights_digest(mine)


def main_melband(unblend) -> None:
    """Mel-Band RoFormer fixtures (reduced model; the kim registry configuration)."""
    with torch.inference_mode():
        cfg = melband_config(**MELBAND_SMALL)
        model, digest = build_melband(unblend, cfg, 5)
        mix = torch.stack([synth_track(0.5, 30), synth_track(0.5, 31)])
        out = model(mix)
        torch.save({"config": cfg, "seed": 5, "weights_digest": digest, "mix": mix, "out": out.clone(),
                    "freq_indices": model.freq_indices.clone(),
                    "num_bands_per_freq": model.num_bands_per_freq.clone()},
                   os.path.join(HERE, "melband_small.pt"))
        cfg = melband_config()
        model, digest = build_melband(unblend, cfg, 6)
        model.configure_inference(sources=["vocals", "other"], samplerate=44100, segment_samples=352800)
        mix = synth_track(1.0, 32)[None]
        out = model(mix)
        torch.save({"config": cfg, "seed": 6, "weights_digest": digest, "mix": mix, "decimate": 5,
                    "sources": ["vocals", "other"], "out": out[..., ::5].clone(), **_summary(out)},
                   os.path.join(HERE, "melband_kim.pt"))


if __name__ == "__main__":
    if len(sys.argv) > 2 and sys.argv[2] == "scnet":
        main_scnet(import_reference(sys.argv[1]))
    elif len(sys.argv) > 2 and sys.argv[2] == "configs":
        main_configs(import_reference(sys.argv[1]))
    elif len(sys.argv) > 2 and sys.argv[2] == "ensemble":
        main_ensemble(import_reference(sys.argv[1]))
    elif len(sys.argv) > 2 and sys.argv[2] == "melband":
        main_melband(import_reference(sys.argv[1]))
    elif len(sys.argv) > 2 and sys.argv[2] == "roformer":
        main_roformer(import_reference(sys.argv[1]))
    else:
        main(sys.argv[1] if len(sys.argv) > 1 else reference_path())
