"""Process-group smoke check (host census, checksum, all-reduce bandwidth) on gloo CPU ranks."""

import socket

import torch

from tests.dist_utils import run_gloo


def _worker(rank, world, expect_nodes):
    from tiny_dsv41_b200.parallel import smoke

    args = smoke.parse_args(["--elements", "4096", "--iterations", "2", "--expected-nodes", str(expect_nodes)])
    report = smoke.run(args, torch.device("cpu"))
    if expect_nodes == 1:
        assert report["ok"], report
        assert report["hosts"] == {socket.gethostname(): world}
        assert report["checksum"] == world * (world + 1) / 2
        assert report["allreduce"]["busbw_gbs"] > 0
    else:
        assert not report["ok"] and "hosts" in report["errors"][0]


def test_smoke_passes_on_one_host():
    run_gloo(_worker, 2, 1)


def test_smoke_reports_a_wrong_host_census():
    run_gloo(_worker, 2, 2)
