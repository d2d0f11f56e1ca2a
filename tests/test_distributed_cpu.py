"""Multi-rank sharding + final gather on CPU ranks (gloo, world size 2), including a rank that
fails before the gather. The per-rank fit is a deterministic stand-in (the product fit needs a
GPU); what is tested is the host logic: shard ranges, global seeds, padding, gather order,
error propagation."""

from __future__ import annotations

import os
import socket
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

from conftest import PKG_DIR, ROOT
from rtgs_b200.image2gs.distributed import shard_range

SCRIPT = textwrap.dedent(
    """
    import datetime, os, sys, json
    sys.path[:0] = [{root!r}, {pkg!r}]
    import torch, torch.distributed as dist
    from rtgs_b200.core.gaussians2d import Gaussians2D
    from rtgs_b200.image2gs.distributed import fit_views_sharded
    from rtgs_b200.image2gs.fit import FitConfig

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=float(os.environ["PG_TIMEOUT"])))
    fail_rank = int(os.environ.get("FAIL_RANK", "-1"))

    def stub_fit(local, config, first_seed):
        if rank == fail_rank:
            raise RuntimeError("injected failure before the gather")
        out, hist = [], []
        for j, img in enumerate(local):
            s = first_seed + j
            g = torch.Generator().manual_seed(s)
            n = config.n_gaussians
            out.append(Gaussians2D(torch.rand(n, 2, generator=g), torch.rand(n, 3, generator=g),
                                   torch.rand(n, 3, generator=g), torch.full((n,), float(s))))
            hist.append({{"seed": s, "rank": rank, "mean": float(img.mean())}})
        return out, hist

    images = [torch.full((4, 4, 3), float(i)) for i in range({n_images})]
    try:
        res, hist = fit_views_sharded(images, FitConfig(n_gaussians=5), seed=10, fit_fn=stub_fit)
        print(json.dumps({{"rank": rank, "seeds": [h["seed"] for h in hist],
                          "ranks": [h["rank"] for h in hist], "means": [h["mean"] for h in hist],
                          "w": [float(g.weight[0]) for g in res], "n": len(res)}}))
    except Exception as exc:
        print(json.dumps({{"rank": rank, "error": type(exc).__name__}}))
        sys.exit(3)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass
    """
)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch(tmp_path: Path, n_images: int, world: int = 2, fail_rank: int = -1, pg_timeout: float = 30.0):
    script = tmp_path / "worker.py"
    script.write_text(SCRIPT.format(root=str(ROOT), pkg=str(PKG_DIR), n_images=n_images))
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), PG_TIMEOUT=str(pg_timeout), FAIL_RANK=str(fail_rank),
                   CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=120)
        except subprocess.TimeoutExpired:
            p.kill()
            out, err = p.communicate()
        outs.append((p.returncode, out, err))
    return outs


def test_shard_ranges_cover_all_items_contiguously():
    for n in range(0, 20):
        for world in (1, 2, 3, 8):
            blocks = [shard_range(n, r, world) for r in range(world)]
            items = [i for s, e in blocks for i in range(s, e)]
            assert items == list(range(n))


@pytest.mark.parametrize("n_images", [4, 5])
def test_two_ranks_gather_every_view_in_order(tmp_path, n_images):
    import json

    outs = _launch(tmp_path, n_images)
    results = []
    for rc, out, err in outs:
        assert rc == 0, err
        results.append(json.loads(out.strip().splitlines()[-1]))
    for res in results:
        assert res["n"] == n_images
        assert res["seeds"] == [10 + i for i in range(n_images)]  # global-index seeds
        assert res["w"] == [float(10 + i) for i in range(n_images)]
        assert res["means"] == [float(i) for i in range(n_images)]
    per = -(-n_images // 2)
    assert results[0]["ranks"] == [0] * per + [1] * (n_images - per)


def test_rank_failing_before_gather_surfaces_as_error_not_hang(tmp_path):
    import json

    outs = _launch(tmp_path, 4, fail_rank=1, pg_timeout=5.0)
    codes = [rc for rc, _, _ in outs]
    assert codes[1] == 3  # the failing rank reports its own error
    assert codes[0] != 0  # the survivor's gather ends with an error instead of waiting forever
    last = outs[0][1].strip().splitlines()
    if last:
        assert "error" in json.loads(last[-1])
