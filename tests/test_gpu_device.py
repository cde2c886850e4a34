"""Device identity on the GPU (bst_device_caps_query): the fields the interceptor's cache key
serialises, as crates/basalto-common/src/hardware.rs:19-57 reads them through the driver."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_device_caps_match_the_runtime():
    import basalto
    c = basalto.device_caps(0)
    p = torch.cuda.get_device_properties(0)
    assert (c["compute_capability_major"], c["compute_capability_minor"]) == (p.major, p.minor)
    assert c["multi_processor_count"] == p.multi_processor_count
    assert c["warp_size"] == 32
    assert c["max_threads_per_block"] == 1024
    assert c["arch"] == f"sm_{p.major}{p.minor}"
    assert c["vendor"] == "nvidia"
    assert c["driver"] and c["driver"] != ""
    assert c["driver_version"] >= 12000
    assert c["name"] == p.name


def test_device_caps_on_b200():
    """The build targets sm_100a: the device the kernels run on is a 148-SM B200."""
    import basalto
    c = basalto.device_caps(0)
    assert (c["compute_capability_major"], c["compute_capability_minor"]) == (10, 0)
    assert c["arch"] == "sm_100"
    assert c["multi_processor_count"] == 148
    assert c["max_registers_per_block"] == 65536
    assert c["max_shared_memory_per_block"] >= 48 * 1024
