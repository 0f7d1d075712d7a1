"""Drop-in ``sdfoam`` module.

The reference's Python (sdfoam_model/scene.py, train.py, extract_mesh.py)
does ``import sdfoam``, whose package imports everything from its compiled
``torch_bindings`` module (torch_bindings/sdfoam/__init__.py.in:29).  With
this package on the path the same import reaches sdfoam_b200's operators:
``create_pipeline`` / ``Pipeline``, ``Triangulation`` /
``TriangulationFailedError``, ``build_aabb_tree``, ``nn``,
``farthest_neighbor``.  The reference's data loader (``BatchFetcher``) and
viewer (``run_with_viewer``) are not part of the tracer and raise an
AttributeError that says so.
"""
from .torch_bindings import *  # noqa: F401,F403
from .torch_bindings import __all__  # noqa: F401
from .torch_bindings import __getattr__  # noqa: F401
