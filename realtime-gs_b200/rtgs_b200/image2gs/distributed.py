"""Multi-GPU Stage-1 fitting: whole images sharded across ranks, one final gather.

Views share no parameters (the reference's batched loss is a per-view sum,
src/rtgs/image2gs/batched.py:142), so rank r fits a contiguous block of images on its own GPU
with no communication during the fit. Per-image initialisation seeds use the GLOBAL image index
(seed + i, as batched.py:66-71), so results do not depend on the number of ranks. The only
collective is one ``all_gather_into_tensor`` of the packed fitted parameters (9 floats per
gaussian: xy, chol, color, weight), padded to the largest shard, plus an object gather of the
small per-view history dictionaries. The process group's timeout bounds every wait: a rank that
fails before the gather makes the others raise instead of hang.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist

from rtgs_b200.core.gaussians2d import Gaussians2D

FitFn = Callable[[list[torch.Tensor], object, int], tuple[list[Gaussians2D], list[dict]]]
PARAMS_PER_GAUSSIAN = 9


def shard_range(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block [start, stop) of ceil(n/world) items for `rank` (last blocks may be short)."""
    per = -(-n_items // world) if n_items else 0
    start = min(rank * per, n_items)
    return start, min(start + per, n_items)


def pack(gaussians: list[Gaussians2D], rows: int, n: int, device) -> torch.Tensor:
    """(rows, n, 9) float32, zero padded past len(gaussians)."""
    out = torch.zeros(rows, n, PARAMS_PER_GAUSSIAN, device=device, dtype=torch.float32)
    for i, g in enumerate(gaussians):
        out[i] = torch.cat([g.xy, g.chol, g.color, g.weight[:, None]], dim=1).to(device, torch.float32)
    return out


def unpack(packed: torch.Tensor) -> list[Gaussians2D]:
    return [Gaussians2D(p[:, 0:2].clone(), p[:, 2:5].clone(), p[:, 5:8].clone(), p[:, 8].clone()) for p in packed]


def fit_views_sharded(
    images: list[torch.Tensor],
    config,
    seed: int = 0,
    *,
    group: dist.ProcessGroup | None = None,
    fit_fn: FitFn | None = None,
    device: torch.device | None = None,
) -> tuple[list[Gaussians2D], list[dict]]:
    """Fit all `images` across the ranks of `group`; every rank returns every view's result.

    ``images`` is the full list; each rank reads only its own block, so entries outside it may be
    None (a rank then never holds the other ranks' images). ``fit_fn(local_images, config,
    seed_of_first)`` defaults to the batched fit engine (``fit_views_batched``). ``device`` is
    where the gathered parameters live (default: the first local image's device; give a CUDA
    device when the local images are host tensors). Without an initialised process group (and
    no ``group``) the calling process is the only rank: it fits every image and gathers nothing.
    """
    if fit_fn is None:
        from rtgs_b200.image2gs.batched import fit_views_batched

        fit_fn = fit_views_batched
    single = group is None and not (dist.is_available() and dist.is_initialized())
    world = 1 if single else dist.get_world_size(group)
    rank = 0 if single else dist.get_rank(group)
    start, stop = shard_range(len(images), rank, world)
    local = images[start:stop]
    results, histories = fit_fn(local, config, seed + start) if local else ([], [])
    n = config.n_gaussians
    per = -(-len(images) // world) if images else 0
    if device is None:
        device = next((im.device for im in local if im is not None), torch.device("cpu"))
    packed = pack(results, per, n, device)
    if single:  # no process group: this process is the only rank and nothing is exchanged
        gathered, all_hist = packed, [histories]
    else:
        gathered = torch.empty(world * per, n, PARAMS_PER_GAUSSIAN, device=device, dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, packed, group=group)
        all_hist: list[list[dict]] = [None] * world  # type: ignore[list-item]
        dist.all_gather_object(all_hist, histories, group=group)
    out, hist = [], []
    for r in range(world):
        s, e = shard_range(len(images), r, world)
        out.extend(unpack(gathered[r * per: r * per + (e - s)]))
        hist.extend(all_hist[r])
    return out, hist
