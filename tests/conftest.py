import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def tiny_foam():
    """Benchmark config 1: 32,768 sites, one 128x128 view (seeded)."""
    from sdfoam_b200 import synthetic as syn
    foam = syn.make_foam("tiny")
    rays, start = syn.camera_rays(foam, syn.views("tiny"), tile=(8, 4))
    return foam, rays, start


@pytest.fixture(scope="session")
def mini_foam():
    """4,096 sites of the tiny mixture and 24x24 rays: fast cases."""
    from sdfoam_b200 import synthetic as syn
    foam = syn.make_foam("tiny", num_points=4096, seed=3)
    cam = syn.look_at((2.2, 1.1, 0.7), fov_deg=40.0, width=24, height=24)
    rays, start = syn.camera_rays(foam, [cam], tile=None)
    return foam, rays, start
