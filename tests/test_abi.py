"""The C-ABI library without a GPU (CPU, no compute calls): it loads, it
exports every function include/nebw.h declares, and with no B200 present it
refuses by name instead of falling back to anything."""

import ctypes as C

import pytest


def test_library_exports_every_declared_symbol():
    import nebw
    declared = nebw.header_functions()
    assert len(declared) >= 25
    lib = C.CDLL(str(nebw.LIB_PATH))
    missing = [f for f in declared if not hasattr(lib, f)]
    assert not missing, f"declared in include/nebw.h but not exported: {missing}"


def test_abi_version():
    import nebw
    assert nebw.lib().nebw_abi_version() == 5


def test_no_gpu_is_an_error_by_name():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import nebw
    with pytest.raises(nebw.NebwError) as e:
        nebw.Device(0)
    assert e.value.code in (1, 2)  # EINVAL (no such device) or ECUDA, never success


def test_null_arguments_refused_without_touching_a_device():
    import nebw
    L = nebw.lib()
    assert L.nebw_model_get_config(None, None) == 1
    assert "null" in L.nebw_last_error().decode()
    assert L.nebw_model_profile(None, 1) == 1
    assert L.nebw_encode_launch_count(None, 0) == -1


def test_oracle_is_not_on_the_product_path():
    """Nothing under the package imports or loads the oracle."""
    from conftest import PKG
    for f in list(PKG.rglob("*.py")) + list(PKG.rglob("*.cu")) + list(PKG.rglob("*.cpp")) + \
            list(PKG.rglob("*.cuh")) + list(PKG.rglob("*.h")):
        text = f.read_text()
        assert "oracle" not in text.replace("oracle/_ref", "").lower() or f.name == "build.py", f
