"""Stage tracing without a GPU: the table arithmetic of fftsparse_b200.trace (the
reference's per-layer stage summary, my_attn_v6_timed.py:44-137), the no-op path
while recording is off, and NVTX-only recording."""
import io

import pytest

from fftsparse_b200 import trace


@pytest.fixture(autouse=True)
def clean():
    trace.disable()
    trace.reset()
    yield
    trace.disable()
    trace.reset()


def test_stage_is_a_no_op_while_off():
    assert not trace.enabled()
    with trace.stage("10_kernel") as s:
        assert s is None
    assert trace.times() == {}


def test_nvtx_only_recording_pushes_ranges_and_records_no_times():
    trace.enable(events=False, nvtx=True)
    with trace.layer(3):
        with trace.stage("4-9_select"):
            pass
    assert trace.times() == {}


def test_table_means_totals_and_layer0_exclusion():
    for ms in (1.0, 3.0):  # layer 0: two calls of each stage
        trace.record(0, "3_mean_pool", ms)
        trace.record(0, "10_kernel", 10 * ms)
    trace.record(1, "3_mean_pool", 4.0)
    trace.record(1, "4-9_select", 1.0)
    trace.record(1, "10_kernel", 30.0)
    t = trace.table()
    assert t["stages"] == ["3_mean_pool", "4-9_select", "10_kernel"]  # schema order
    assert t["per_layer"][0] == {"3_mean_pool": 2.0, "4-9_select": 0.0, "10_kernel": 20.0}
    assert t["layer_total"] == {0: 22.0, 1: 35.0}
    assert t["mean"] == {"3_mean_pool": 3.0, "4-9_select": 0.5, "10_kernel": 25.0}
    assert t["mean_excl_layer0"] == {"3_mean_pool": 4.0, "4-9_select": 1.0, "10_kernel": 30.0}
    buf = io.StringIO()
    trace.summary(file=buf)
    text = buf.getvalue()
    assert "10_kernel" in text and "22.0000" in text and "35.0000" in text


def test_unknown_stage_names_follow_the_schema():
    trace.record(2, "11_gather", 0.5)
    trace.record(2, "10_kernel", 1.5)
    assert trace.table()["stages"] == ["10_kernel", "11_gather"]


def test_layer_context_restores_the_previous_layer():
    trace.enable(events=False, nvtx=True)
    with trace.layer(5):
        with trace.layer(7):
            assert trace._layer[0] == 7
        assert trace._layer[0] == 5
    assert trace._layer[0] == 0
