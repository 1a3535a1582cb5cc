"""Shared pytest configuration: the ``gpu`` marker and common fixtures."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")


@pytest.fixture
def rng() -> np.random.Generator:
    """A seeded generator (seed 1234, as the reference's own test suite uses)."""
    return np.random.default_rng(1234)


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN, name)) as f:
        return {k: f[k] for k in f.files}


def assert_parity(ours: np.ndarray, ref: np.ndarray, rel: float, what: str = "") -> None:
    """The parity metric: ``max|d| <= rel * max|ref|`` and ``||d||_2 <= rel * ||ref||_2``.

    Elementwise ``rtol`` is not used: any reordering of fp32 sums moves near-zero entries by
    more than a relative 1e-4 of themselves, while the tensor as a whole agrees.
    """
    ours = np.asarray(ours, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert ours.shape == ref.shape, f"{what}: shape {ours.shape} != {ref.shape}"
    assert np.all(np.isfinite(ours)), f"{what}: non-finite values"
    d = ours - ref
    max_ref = float(np.max(np.abs(ref))) if ref.size else 0.0
    norm_ref = float(np.linalg.norm(ref))
    max_err = float(np.max(np.abs(d))) if d.size else 0.0
    norm_err = float(np.linalg.norm(d))
    assert max_err <= rel * max_ref + 1e-30, f"{what}: max err {max_err:.3e} > {rel} * {max_ref:.3e}"
    assert norm_err <= rel * norm_ref + 1e-30, (
        f"{what}: norm err {norm_err:.3e} > {rel} * {norm_ref:.3e}"
    )


def ill_conditioned(ref_grad: np.ndarray, rel: float) -> np.ndarray:
    """Entries whose reference gradient is below ``rel * max|g|``.

    Adam's first update there is ``lr * g / (|g| + eps)``: at the parity tolerance neither
    the sign nor the size of such a ``g`` is determined, so neither is the update. An fp32
    computation matching the gradients to ``rel`` can still move these entries by up to
    ``2 lr``; later steps inherit the difference through the parameter and the moments.
    """
    g = np.abs(np.asarray(ref_grad, dtype=np.float64))
    return g < rel * (g.max() if g.size else 0.0)


def assert_update_parity(ours: np.ndarray, ref: np.ndarray, ill: np.ndarray, rel: float,
                         what: str = "", max_ill_fraction: float = 0.5) -> None:
    """Post-optimizer parameters: both criteria over the entries whose gradients are
    determined at the tolerance (``ill_conditioned``), relative to the whole reference
    tensor. Excluded are e.g. the key slice of the QKV bias, whose exact gradient is zero
    (softmax is invariant to a per-row shift), so that Adam moves it by the sign of rounding
    noise in the reference and here alike."""
    ours = np.asarray(ours, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert ours.shape == ref.shape, f"{what}: shape {ours.shape} != {ref.shape}"
    assert float(ill.mean()) <= max_ill_fraction, f"{what}: {ill.mean():.2%} ill-conditioned"
    well = ~ill
    d = (ours - ref)[well]
    if not d.size:
        return
    assert np.linalg.norm(d) <= rel * np.linalg.norm(ref) + 1e-30, (
        f"{what}: norm err {np.linalg.norm(d):.3e} > {rel} * {np.linalg.norm(ref):.3e}"
    )
    err = float(np.abs(d).max())
    assert err <= rel * float(np.abs(ref).max()) + 1e-30, (
        f"{what}: max err {err:.3e} over well-conditioned entries > {rel} * "
        f"{np.abs(ref).max():.3e}"
    )


def assert_zero_gradient(ours: np.ndarray, scale: float, rel: float, what: str = "") -> None:
    """A gradient that is exactly zero in exact arithmetic: the bias of a convolution that
    feeds a batch norm (the norm removes any per-channel shift). Both the reference and this
    build hold rounding noise there, so the check is absolute: every entry within
    ``rel * scale``, ``scale`` the largest entry of the same layer's weight gradient."""
    ours = np.asarray(ours, dtype=np.float64)
    assert np.all(np.isfinite(ours)), f"{what}: non-finite values"
    err = float(np.abs(ours).max()) if ours.size else 0.0
    assert err <= rel * scale, f"{what}: |g| {err:.3e} > {rel} * {scale:.3e}"
