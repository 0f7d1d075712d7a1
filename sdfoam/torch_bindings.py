"""``sdfoam.torch_bindings``: the reference's compiled operator module
(torch_bindings/torch_bindings.cpp:69-84, pipeline_bindings.cpp:799-860,
triangulation_bindings.cpp:219-248) answered by sdfoam_b200."""
import sdfoam_b200 as _impl
from sdfoam_b200 import *  # noqa: F401,F403

__all__ = list(_impl.__all__)

# Names of the reference module that belong to its data loader or its
# OpenGL viewer, outside the tracer this package replaces.
_NOT_PROVIDED = {
    "BatchFetcher": "the reference's threaded ray/RGB batch loader (src/utils/batch_fetcher.cpp); "
                    "index the ray tensors on the GPU instead",
    "run_with_viewer": "the reference's OpenGL viewer (src/viewer); there is no graphics stack here",
}


def __getattr__(name):
    if name in _NOT_PROVIDED:
        raise AttributeError(f"sdfoam.{name} is not provided by sdfoam_b200: {_NOT_PROVIDED[name]}")
    raise AttributeError(f"module 'sdfoam' has no attribute {name!r}")
