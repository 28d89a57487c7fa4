"""Host-side helpers of bench.py: the NCCL share of the push by load kind, the exchange
summary's NVLink fraction, and the GPU topology record (parsed from nvidia-smi's output)."""
import os
import sys
import types

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _args(share="auto"):
    return types.SimpleNamespace(push_nccl_share=share)


def test_push_share_only_where_the_exchange_is_the_long_leg():
    assert bench.push_share(_args(), 4) == 0.0  # hash-bound loads: copy engines alone
    assert bench.push_share(_args(), 4, exchange_bound=True) == 0.3
    assert bench.push_share(_args(), 2, exchange_bound=True) == 0.0
    assert bench.push_share(_args(), 8, exchange_bound=True) == 0.0
    assert bench.push_share(_args("0.45"), 2) == 0.45
    assert bench.push_share(_args("3"), 4) == 1.0 and bench.push_share(_args("-1"), 4) == 0.0


def test_exchange_summary_fraction_of_nvlink():
    s = bench.exchange_summary("push", 26.6e9, 70.0, 63.9, 0.3)
    assert s["gbs_per_rank"] == pytest.approx(26.6e9 / 63.9 / 1e6, rel=1e-3)
    assert s["frac_of_nvlink_900"] == pytest.approx(s["gbs_per_rank"] / 900, rel=1e-3)
    assert "0.3" in s["mode"] and "NCCL" in s["mode"]
    assert bench.exchange_summary("nccl", 1e9, 5.0, 0.0)["gbs_per_rank"] == 0.0


def test_gpu_topology_parses_topo_matrix(monkeypatch):
    topo = ("\t\x1b[4mGPU0\tGPU1\tGPU2\tNIC0\tCPU Affinity\tNUMA Affinity\tGPU NUMA ID\x1b[0m\n"
            "GPU0\t X \tNV18\tNV18\tPIX\t0-31\t0\t\tN/A\n"
            "GPU1\tNV18\t X \tNV18\tSYS\t0-31\t0\t\tN/A\n"
            "GPU2\tNV18\tNV18\t X \tSYS\t32-63\t1\t\tN/A\n"
            "NIC0\tPIX\tSYS\tSYS\t X \n\nLegend:\n  X    = Self\n")
    ids = "0, 00000000:18:00.0\n1, 00000000:2A:00.0\n2, 00000000:9A:00.0\n"

    def fake_run(cmd, **kw):
        return types.SimpleNamespace(stdout=ids if "--query-gpu=index,pci.bus_id" in cmd else topo)

    monkeypatch.setattr(bench.subprocess, "run", fake_run)
    t = bench.gpu_topology(2)
    assert t["pci_bus_ids"] == ["00000000:18:00.0", "00000000:2A:00.0"]
    assert set(t["topo"]) == {"GPU0", "GPU1"}
    assert t["topo"]["GPU0"]["gpus"] == ["X", "NV18"]
    assert t["topo"]["GPU0"]["nics"] == {"NIC0": "PIX"} and t["topo"]["GPU1"]["numa"] == "0"


def test_gpu_topology_without_nvidia_smi(monkeypatch):
    def missing(cmd, **kw):
        raise FileNotFoundError("nvidia-smi")

    monkeypatch.setattr(bench.subprocess, "run", missing)
    assert "error" in bench.gpu_topology(4)
