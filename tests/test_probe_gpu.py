"""Domain probes on the GPU: one cooperative launch each, bounded waits, consistent maps.

When L2D_PROBE_DUMP names a directory, the raw latency samples are written there as JSON so the
near/far distributions can be inspected off the GPU box."""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402

DUMP = os.environ.get("L2D_PROBE_DUMP")


@pytest.fixture(scope="module")
def sm_map():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    m, extra = L.get_map_smid2side(0, with_raw=True)
    if DUMP:
        os.makedirs(DUMP, exist_ok=True)
        with open(os.path.join(DUMP, "probe_sm_raw.json"), "w") as f:
            json.dump({"map": m, **extra, "device": L.device_info(0)}, f)
    assert extra["status"] == 0, extra["error"]
    return m, extra["report"]


def test_sm_map_two_domains(sm_map):
    m, rep = sm_map
    n = L.num_sms(0)
    assert len(m) == n and set(m) == {0, 1} and m[0] == 0
    assert rep["domain_sms"][0] + rep["domain_sms"][1] == n
    assert rep["far_cycles"] > rep["near_cycles"] and rep["separation"] >= 3
    assert rep["device_status"] == 0


def test_sm_map_is_stable(sm_map):
    m, _ = sm_map
    assert L.get_map_smid2side(0) == m


def test_addr_model_consistent(sm_map):
    m, _ = sm_map
    raw = torch.empty(66 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % (2 * 1024 * 1024)
    base = raw.data_ptr() + off
    (mask, attr), extra = L.get_map_memory_attr(base, 64 * 1024 * 1024, m, 0, with_raw=True)
    if DUMP:
        with open(os.path.join(DUMP, "probe_addr_raw.json"), "w") as f:
            json.dump({"mask": mask, "attr": attr, **extra}, f)
    assert extra["status"] == 0, extra["error"]
    rep = extra["report"]
    assert len(attr) == 32
    assert rep["mask_agreement"] >= 0.95 and rep["attr_agreement"] >= 0.75
    # A second allocation of the same device gives the same within-page mask.
    raw2 = torch.empty(10 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    off2 = (-raw2.data_ptr()) % (2 * 1024 * 1024)
    (mask2, attr2) = L.get_map_memory_attr(raw2.data_ptr() + off2, 8 * 1024 * 1024, m, 0)
    assert mask2 == mask and len(attr2) == 4


def test_probe_rejects_bad_arguments(sm_map):
    m, _ = sm_map
    raw = torch.empty(4 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(L.L2DError):
        L.get_map_memory_attr(raw.data_ptr() + 128, 2 * 1024 * 1024, m, 0)  # misaligned base
    with pytest.raises(L.L2DError):
        L.get_map_memory_attr(raw.data_ptr(), 2 * 1024 * 1024, m[:-1], 0)  # map of the wrong size


def test_probe_timeout_is_reported_not_hung(sm_map):
    """A 1 ms bound on every device wait: the probe either finishes or returns a timeout status;
    the context stays usable either way."""
    m, extra = L.get_map_smid2side(0, timeout_ms=1, with_report=True)
    assert extra["status"] in (0, -4, -6)
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum()) == 8.0
