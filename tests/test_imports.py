"""Port of the reference's import tests (tests/test_imports.py:3-12)."""


def test_imports():
    from gdn2_package import gdn2_pallas_forward_trainable, gdn2_pallas_forward
    assert gdn2_pallas_forward_trainable is not None
    assert gdn2_pallas_forward is not None


def test_version():
    import gdn2_package
    assert hasattr(gdn2_package, "__version__")


def test_module_constants():
    from gdn2_package import gdn2_fwd
    assert (gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.MB, gdn2_fwd.CLIP) == (256, 128, 16, 1e4)
