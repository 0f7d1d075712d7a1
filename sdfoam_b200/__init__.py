"""sdfoam_b200 -- B200-native Voronoi-foam tracer behind SDFoam's operator surface.

``import sdfoam_b200 as sdfoam`` gives the names the reference's ``sdfoam``
module exposes for the tracing path (torch_bindings/pipeline_bindings.cpp:
799-860): ``create_pipeline`` returning a ``Pipeline`` with ``trace_forward`` /
``trace_backward``, plus ``build_aabb_tree``, ``nn`` and ``farthest_neighbor``
(triangulation_bindings.cpp:239-248), ``Triangulation`` /
``TriangulationFailedError`` (the Delaunay adjacency rebuild,
triangulation_bindings.cpp:219-237) and ``sort_points`` (its site order,
aabb_tree.cu:62-190).  ``sdfoam_b200.render.TraceRays`` is the drop-in for
``sdfoam_model.render.TraceRays``.  All compute runs in libsdfoam_b200.so
(include/sdfoam_b200.h); there is no CPU fallback.
"""
from .pipeline import Pipeline, create_pipeline, pipeline_registry  # noqa: F401
from .spatial import build_aabb_tree, farthest_neighbor, nn, sort_points  # noqa: F401
from .triangulation import Triangulation, TriangulationFailedError  # noqa: F401

__all__ = ["Pipeline", "create_pipeline", "pipeline_registry", "build_aabb_tree", "nn", "farthest_neighbor",
           "sort_points", "Triangulation", "TriangulationFailedError"]
