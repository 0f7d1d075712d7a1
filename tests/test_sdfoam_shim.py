"""The drop-in ``sdfoam`` package: ``import sdfoam`` as the reference's
Python does (sdfoam_model/scene.py:8) reaches sdfoam_b200's operators."""
import pytest


def test_import_sdfoam_reaches_the_b200_operators():
    import sdfoam
    import sdfoam.torch_bindings as tb
    import sdfoam_b200

    for name in ("create_pipeline", "Pipeline", "Triangulation", "TriangulationFailedError", "build_aabb_tree",
                 "nn", "farthest_neighbor"):
        assert getattr(sdfoam, name) is getattr(sdfoam_b200, name)
        assert getattr(tb, name) is getattr(sdfoam_b200, name)
    assert set(sdfoam.__all__) == set(sdfoam_b200.__all__)
    with pytest.raises(AttributeError, match="not provided by sdfoam_b200"):
        sdfoam.BatchFetcher
    with pytest.raises(AttributeError, match="no attribute"):
        sdfoam.no_such_name
