"""lyth-probe's checks, restated (lyth_b200.probe), on the host: the ncu CSV parser and the
derived-vs-measured verdicts (crates/lyth-probe/src/ncu.rs:690-838, its own test cases), the
machine-file check (crates/lyth-probe/src/machine.rs:352-420) against the reference's own machine
fixtures, and the derived cost of every in-scope example against the intensity its source
declares (the compiler refuses a declaration that disagrees with the derived one)."""
import glob
import json
import os

import pytest

from lyth_b200 import examples as ex
from lyth_b200 import probe as p

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CSV = '''"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"
"0","k_integrate(int, int)","dram__bytes.sum","Mbyte","4.75"
"0","k_integrate(int, int)","gpu__time_duration.sum","usecond","120.5"
"1","k_propagate(int)","dram__bytes.sum","Mbyte","2.00"
'''
SPLIT = '''"Kernel Name","Metric Name","Metric Unit","Metric Value"
"k_integrate(int, int)","dram__bytes.sum","byte","2.508.800"
"k_integrate(int, int)","dram__bytes_op_read.sum","byte","2.508.800"
"k_integrate(int, int)","dram__bytes_op_write.sum","byte","0"
'''


def test_named_kernel_and_unit_scale():
    t = p.parse_ncu(CSV, "k_integrate")
    assert t["bytes"] == 4.75e6 and t["launches"] == 1 and "k_integrate" in t["kernel"]


def test_folding_names_what_it_folded():
    t = p.parse_ncu(CSV)
    assert t["bytes"] == 6.75e6 and "+" in t["kernel"]


def test_missing_kernel_lists_what_is_there():
    with pytest.raises(p.NcuError, match="k_integrate"):
        p.parse_ncu(CSV, "k_nope")


def test_confirmed_inflated_absorbed():
    t = p.parse_ncu(CSV, "k_integrate")
    assert p.compare(29.0, 163_903, t, "all", 0.05)["verdict"] == "confirmed"
    assert p.compare(8.0, 163_903, t, "all", 0.05)["verdict"] == "inflated"
    assert p.compare(200.0, 163_903, t, "all", 0.05)["verdict"] == "absorbed"


def test_separators():
    assert p.parse_value("1,234.5", "Mbyte") == 1234.5e6
    assert p.parse_value("1.234,5", "Mbyte") == 1234.5e6
    assert p.parse_value("2.508.800", "byte") == 2_508_800.0
    assert p.parse_value("2,508,800", "byte") == 2_508_800.0
    assert p.parse_value("4.750", "byte") == 4750.0
    assert p.parse_value("4.750", "Mbyte") == 4.75e6
    assert p.parse_value("n/a", "") is None
    with pytest.raises(p.NcuError):
        p.parse_value("4.75", "furlongs")


def test_read_only_measurement_confirms_the_read_half():
    t = p.parse_ncu(SPLIT)
    assert t["read"] == 2_508_800.0 and t["write"] == 0.0
    assert p.compare(29.0, 166_700, t, "all", 0.05)["verdict"] == "absorbed"
    assert p.compare(15.0, 166_700, t, "read", 0.05)["verdict"] == "confirmed"


def test_no_split_refuses_a_direction():
    t = p.parse_ncu(CSV, "k_integrate")
    with pytest.raises(p.NcuError, match="dram__bytes_op_read"):
        p.compare(15.0, 166_700, t, "read", 0.05)


def test_reference_captures_parse_locale_safely():
    # the reference's own sm_120 captures, dots grouping the digits
    want = {"k_integrate": (2_508_544, 2_508_544, 0), "k_propagate": (1_239_296, 1_230_336, 8_960),
            "saxpy-lyth": (182_320_640, 134_222_848, 48_097_792)}
    for name, (tot, rd, wr) in want.items():
        path = glob.glob(os.path.join(G, "ncu", name + "*.csv"))[0]
        t = p.parse_ncu(open(path).read())
        assert (t["bytes"], t["read"], t["write"]) == (tot, rd, wr), name
    t = p.parse_ncu(open(glob.glob(os.path.join(G, "ncu", "rmsnorm*.csv"))[0]).read())
    assert t["bytes"] == 118_885_888 and t["metrics"]["lts__t_bytes.sum"] == 214_566_432
    # the reference's saxpy at n = 2^24 (12 B/elem derived): L2 confirms, DRAM absorbs the writes
    t = p.parse_ncu(open(glob.glob(os.path.join(G, "ncu", "saxpy-lyth*.csv"))[0]).read())
    l2 = p.parse_ncu(open(glob.glob(os.path.join(G, "ncu", "saxpy-lyth*.csv"))[0]).read(), level="l2")
    assert p.compare(12.0, 1 << 24, l2, "all", 0.02)["verdict"] == "confirmed"
    assert p.compare(8.0, 1 << 24, t, "read", 0.02)["verdict"] == "confirmed"
    assert p.compare(4.0, 1 << 24, t, "write", 0.02)["verdict"] == "absorbed"


def load(name):
    with open(os.path.join(G, "machine", name)) as f:
        return json.load(f)


def test_machine_check_on_the_reference_fixtures():
    meas = load("meas-sm_120-2026-09-14.json")
    lie = p.check_machine(load("sm_120-lie.json"), meas)
    assert lie["verdict"] == "fail" and any("500.00" in m for m in lie["mismatches"])
    stale = p.check_machine(load("sm_120-stale-ridge.json"), meas)
    assert stale["verdict"] == "fail" and any("42.88" in m and "drifts" in m for m in stale["mismatches"])
    honest = {"schema": p.MACHINE_SCHEMA, "id": "sm_120", "peak_tflops": 15.37,
              "levels": [{"name": "dram", "bandwidth_gbs": 358.43}], "ridge_flop_per_byte": {"fp32": 42.88}}
    assert p.check_machine(honest, meas)["verdict"] == "pass"
    assert abs(p.ridge_fp32(honest) - 42.88) < 0.05
    with pytest.raises(ValueError, match="machine id"):
        p.check_machine(dict(honest, id="sm_100a"), meas)
    bad = dict(meas, levels=[{"name": "dram", "bandwidth_gbs": 400.0, "runs": [350.0, 358.0, 360.0]}])
    assert "not self-consistent" in p.check_machine(honest, bad)["mismatches"][0]


def test_the_b200_machine_file():
    path = p.MACHINE_FILE
    m = json.load(open(path))
    assert m["schema"] == p.MACHINE_SCHEMA and m["id"] == "sm_100a"
    assert p.accepts(m, "sm_100a") and p.accepts(m, "sm_120") and not p.accepts(m, "sm_90")
    dram = next(lv for lv in m["levels"] if lv["name"] == "dram")
    assert dram["bandwidth_gbs"] > 1000 and m["sm_count"] == 148
    assert m["smem_banks"] == 32 and m["smem_bank_bytes"] == 4
    assert abs(m["ridge_flop_per_byte"]["fp32"] - p.ridge_fp32(m)) / p.ridge_fp32(m) < 0.005
    meas_path = os.path.join(os.path.dirname(path), "meas-sm_100a.json")
    assert p.check_machine(m, json.load(open(meas_path)))["verdict"] == "pass"


# the `intensity` line each example declares (examples/*.lyth)
DECLARED = {"saxpy": 0.1667, "axpby": 0.25, "lerp": 0.25, "horner": 0.75, "copy2d": 0.0, "transpose": 0.0,
            "transpose_tiled": 0.0, "sum": 0.25, "dot": 0.25, "max_of": 0.0, "min_of": 0.0, "hadamard_q": 0.25,
            "gate_q": 0.875, "cu_q": 0.4375, "swap_q": 0.0}


@pytest.mark.parametrize("name", sorted(DECLARED))
def test_derived_intensity_matches_the_declaration(name):
    c = p.derive_cost(ex.IN_SCOPE[name]())
    assert abs(c["intensity"] - DECLARED[name]) < 5e-4, c


def test_derived_bytes_per_element():
    assert p.derive_cost(ex.saxpy())["bytes"] == 12
    assert p.derive_cost(ex.horner())["bytes"] == 8
    assert p.derive_cost(ex.transpose(True))["bytes"] == 8
    assert p.derive_cost(ex.reduction("dot"))["bytes"] == 8
    assert p.derive_cost(ex.gate_q())["bytes"] == 32     # per pair: 16 B per amplitude
    assert p.derive_cost(ex.cu_q())["bytes"] == 64       # per quad
    with pytest.raises(ValueError):
        p.derive_cost(ex.matmul())
