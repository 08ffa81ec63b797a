"""Host-side pieces of bench.py that only GPU runs exercise end to end: the
clock summary of a timed window, the exp-unit roofline arithmetic, the
sub-record switch and the workload table.  No GPU needed."""
import types

import pytest

import bench


def sampler_with(samples, max_mhz=1965):
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.samples = samples
    s.thread = None
    s.max_mhz = max_mhz
    return s


def test_clock_window_median_and_reasons():
    # (host time, SM MHz, clock-event reason bits, power W)
    samples = [(0.0, 1000, 0, 100.0), (1.0, 1965, 0, 500.0), (1.1, 1900, bench.REASON_BITS["sw_power_cap"], 900.0),
               (1.2, 1965, 0, 950.0), (3.0, 500, bench.REASON_BITS["hw_slowdown"], 90.0)]
    c = sampler_with(samples).window(0.9, 1.3)
    assert c["sm_mhz"] == 1965 and c["samples"] == 3 and c["sm_max_mhz"] == 1965
    assert c["reasons"] == ["sw_power_cap"] and c["power_w_max"] == 950.0


def test_clock_window_shorter_than_one_period_takes_the_next_sample():
    c = sampler_with([(0.0, 1000, 0, 1.0), (2.0, 1800, 0, 1.0)]).window(1.0, 1.001)
    assert c["sm_mhz"] == 1800 and c["samples"] == 1
    assert sampler_with([]).window(0.0, 1.0) is None


def test_mufu_roofline():
    # 148 SMs x 16 ex2/clk at 1965 MHz = 4653 Gexp/s; 4.653e9 exps in 1 ms is all of it
    r = bench.mufu_roofline(4.65312e9, 1.0, {"sm_mhz": 1965.0}, 148)
    assert r["unit"] == "Gexp/s" and abs(r["peak"] - 4653.12) < 1e-6 and abs(r["frac"] - 1.0) < 1e-6
    # no clock record: the nominal maximum clock
    assert abs(bench.mufu_roofline(1e9, 1.0, None, 148)["peak"] - 4653.12) < 1e-6


def test_sub_records_only_on_the_default_workload():
    a = types.SimpleNamespace(workload="attention", shape=None, no_sub=False)
    assert bench.sub_records_enabled(a)
    assert not bench.sub_records_enabled(types.SimpleNamespace(workload="attention", shape="1,1,128,64", no_sub=False))
    assert not bench.sub_records_enabled(types.SimpleNamespace(workload="softmax", shape=None, no_sub=False))
    assert not bench.sub_records_enabled(types.SimpleNamespace(workload="attention", shape=None, no_sub=True))


def test_sub_records_are_the_baseline_configs():
    keys = {k: w for k, w, *_ in bench.SUB_RECORDS}
    assert keys == {"attention_cfg2": "attention-cfg2", "attention_cfg4": "attention-cfg4", "softmax_cfg5": "softmax"}
    assert bench.WORKLOADS["attention"][:4] == (16, 32, 4096, 128)
    assert bench.WORKLOADS["attention-cfg2"][:5] == (8, 16, 1024, 64, "float16")
    assert bench.WORKLOADS["attention-cfg4"][:6] == (1, 32, 32768, 128, "bfloat16", 0.5)
    assert bench.WORKLOADS["softmax"][:2] == (65536, 1024) and bench.WORKLOADS["softmax"][5] == 2.0
    assert bench.WORKLOADS["attention-cfg1"][:5] == (2, 4, 128, 64, "float32")


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_every_workload_has_a_runner(name):
    fn = bench.RUNNERS.get(name, bench.run_attention)
    assert callable(fn)
    if name.startswith("softmax"):
        assert fn is bench.run_softmax


def test_softmax_kernel_name_follows_the_dispatch_rule():
    # pmkl_warp_softmax_fwd: fp32 rows of multiples of 4 -> 16-byte vectors;
    # other dtypes with rows of multiples of 8 -> 8-element vectors; else general
    assert bench.softmax_kernel_name(4, 1024) == "softmax_vec_kernel"
    assert bench.softmax_kernel_name(4, 1023) == "softmax_gen_kernel"
    assert bench.softmax_kernel_name(2, 1024) == "softmax_vec8_kernel"
    assert bench.softmax_kernel_name(2, 1020) == "softmax_gen_kernel"


def test_extra_workloads_have_runners():
    for name in ("softmax-gen", "attention-bwd-fp32", "softmax-bf16", "attention-bwd"):
        assert name in bench.WORKLOADS and name in bench.RUNNERS
    # the reference arm's attention-bwd family shares one worker
    assert bench.WORKLOADS["attention-bwd-fp32"][4] == "float32"
