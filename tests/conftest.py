"""Shared pytest setup: paths, the `gpu` marker, and fixtures for synthetic containers."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_ROOT = REPO / "turbo-winfare-dense_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def built_lib():
    """Builds (incrementally) and returns the path of libg4dense_b200.so."""
    from g4dense_b200 import build
    return build.build()


@pytest.fixture(scope="session")
def config0(tmp_path_factory):
    """BASELINE config 0 containers (seed 0 target, seed 1 drafter) plus a zero-mean variant."""
    from g4dense_b200 import container as C
    d = tmp_path_factory.mktemp("config0")
    paths = {
        "target": C.write_container(d / "target.g4dense", C.CONFIG0_TARGET, seed=0),
        "draft": C.write_container(d / "draft.g4dense", C.CONFIG0_DRAFT, seed=1),
        "target_centered": C.write_container(d / "target_c.g4dense", C.CONFIG0_TARGET, seed=0, centered=True),
        "draft_centered": C.write_container(d / "draft_c.g4dense", C.CONFIG0_DRAFT, seed=1, centered=True),
    }
    paths["near_draft"] = C.perturbed_copy(paths["target"], d / "near_draft.g4dense", C.CONFIG0_TARGET, 0.0,
                                           seed=C.NEAR_DRAFT_SEED, embed_frac=C.NEAR_DRAFT_EMBED_FRAC)
    return paths


@pytest.fixture(scope="session")
def geom31(tmp_path_factory):
    from g4dense_b200 import container as C
    d = tmp_path_factory.mktemp("geom31")
    spec = C.GEOM31_TEST
    return {
        "baseline": C.write_container(d / "g31.g4dense", spec, seed=5),
        "centered": C.write_container(d / "g31_c.g4dense", spec, seed=5, centered=True),
    }
