"""Sharded, reshardable checkpoints.

Layout of one checkpoint (a directory per step)::

    <root>/step_00000100/
        manifest.json              config, topology, step, seed, tensor index
        shard_tp{t}_pp{p}.pt       {global name: local tensor} for one (tp, pp) cell,
                                   model weights plus optimizer state
        COMPLETE                   written last by rank 0: the checkpoint is whole

``save(..., background=True)`` returns after the tensors are copied to host
memory and writes the files from a thread (see :class:`PendingSave`).

Each (tp, pp) cell is written by its data-parallel rank 0 (DP replicas hold
identical weights and optimizer state). Tensors are keyed by their GLOBAL
name - the parameter name in the full single-process model (via
``ref_param_name``) prefixed with ``model/``, ``master/``, ``exp_avg/`` or
``exp_avg_sq/`` - and the manifest records, per global name, the full shape
and how it is split across TP ranks (dimension, or ``null`` when
replicated) and which pipeline stage holds it. Because initialisation and
naming are decomposition-invariant, loading into a different TP/PP layout is
a concatenate-then-slice: a checkpoint written at tp=2 x pp=2 loads at tp=1 or
tp=4 unchanged. Data needs no state: batches are a pure function of (seed,
step, dp rank).

The reference has no checkpointing; this format is new.
"""

from __future__ import annotations

import argparse
import datetime
import hashlib
import json
import os
import shutil
import threading
from typing import Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from ..models.layers import ColumnParallelLinear, RowParallelLinear

STATE_KINDS = ("master", "exp_avg", "exp_avg_sq")


def split_dim(model: nn.Module, local_name: str) -> Optional[int]:
    """TP split dimension of a parameter (None when replicated)."""
    owner = model.get_submodule(local_name.rsplit(".", 1)[0]) if "." in local_name else model
    leaf = local_name.rsplit(".", 1)[-1]
    if isinstance(owner, ColumnParallelLinear):
        return 0
    if isinstance(owner, RowParallelLinear) and leaf == "weight":
        return 1
    return None


def _global_name(model: nn.Module, name: str) -> str:
    fn = getattr(model, "ref_param_name", None)
    return fn(name) if fn else name


def _optimizer_state(opt, params):
    """Per-parameter fp32 state tensors: master weights and Adam moments when
    the optimizer keeps them; ``step`` as a float. Sharded optimizer state
    (FusedDPAdam) is gathered over the DP group - collective."""
    from ..optim.fused_dp import FusedDPAdam
    from ..optim.precision import MasterWeightOptimizer

    out = {}
    step = 0.0
    if isinstance(opt, FusedDPAdam):
        for name, p in params:
            out[name] = opt.full_state(p)
        return out, float(opt._step)
    if isinstance(opt, MasterWeightOptimizer):
        by_param = dict(zip([id(p) for p in opt.model_params], opt.master_params))
        for name, p in params:
            m = by_param.get(id(p))
            if m is None:
                continue
            st = opt.inner.state.get(m, {})
            out[name] = {"master": m}
            if st:
                out[name]["exp_avg"] = st["exp_avg"]
                out[name]["exp_avg_sq"] = st["exp_avg_sq"]
                step = float(st["step"])
    elif isinstance(opt, torch.optim.Optimizer):
        for name, p in params:
            st = opt.state.get(p, {})
            if st:
                out[name] = {"exp_avg": st["exp_avg"], "exp_avg_sq": st["exp_avg_sq"]}
                step = float(st["step"])
    return out, step


class PendingSave:
    """Handle of a checkpoint being written in the background. ``wait()``
    blocks until this rank's part is on disk (rank 0: until the whole
    checkpoint is marked COMPLETE) and re-raises a writer error."""

    def __init__(self, path: str, thread: Optional[threading.Thread] = None):
        self.path = path
        self._thread = thread
        self.error: Optional[BaseException] = None

    def wait(self) -> str:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self.error is not None:
            raise RuntimeError(f"checkpoint {self.path} failed") from self.error
        return self.path

    def done(self) -> bool:
        return self._thread is None or not self._thread.is_alive()


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def _write_shard(tensors: Dict[str, torch.Tensor], shard_file: str) -> None:
    """The shard, then its SHA-256 next to it (``<shard>.sha256``)."""
    torch.save(tensors, shard_file)
    with open(shard_file + ".sha256", "w") as f:
        f.write(_sha256(shard_file) + "\n")


def verify_shard(shard_file: str) -> bool:
    """True when the shard matches its recorded SHA-256 (or none was recorded)."""
    rec = shard_file + ".sha256"
    if not os.path.exists(rec):
        return True
    with open(rec) as f:
        return f.read().strip() == _sha256(shard_file)


def _snapshot(t: torch.Tensor, background: bool) -> torch.Tensor:
    """Host copy of ``t``; a CPU tensor is copied only when the file is
    written in the background (training would otherwise change it)."""
    c = t.detach().cpu()
    return c.clone() if background and c.data_ptr() == t.data_ptr() else c


def _write_manifest(path, gathered, step, seed, opt_step, config, tp, pp, dp, extra) -> None:
    merged = {}
    for part in gathered:
        if part and part.get("index"):
            merged.update(part["index"])
    manifest = {
        "format": "dstraining_b200/sharded-v1",
        "step": step,
        "seed": seed,
        "optimizer_step": opt_step,
        "config": dict(vars(config)),
        "topology": {"tp": tp.world, "pp": pp.world, "dp": dp.world},
        "tensors": merged,
        "extra": extra or {},
    }
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)


def save(root: str, step: int, model: nn.Module, opt, tp, pp, dp, config, seed: int, extra: Optional[dict] = None,
         background: bool = False, timeout_s: float = 1800.0):
    """Write a checkpoint of every rank's shard (collective: call on all ranks).

    ``background=False`` returns the checkpoint path once it is complete.
    ``background=True`` does the collective part (gathering sharded optimizer
    state, exchanging the tensor index) and copies every tensor to host memory
    before returning a :class:`PendingSave`; the files are then written by a
    thread, and rank 0 marks the checkpoint COMPLETE after every writer has
    reported through the rendezvous store - so training continues while the
    disk writes run. Call ``wait()`` before the next save and before exit."""
    path = os.path.join(root, f"step_{step:08d}")
    rank = dist.get_rank() if dist.is_initialized() else 0
    if rank == 0:
        os.makedirs(path, exist_ok=True)
    if dist.is_initialized():
        dist.barrier()
    params = list(model.named_parameters())
    state, opt_step = _optimizer_state(opt, params)
    index: Dict[str, dict] = {}
    tensors: Dict[str, torch.Tensor] = {}
    for name, p in params:
        g = _global_name(model, name)
        d = split_dim(model, name)
        full = list(p.shape)
        if d is not None:
            full[d] *= tp.world
        index[f"model/{g}"] = {"shape": full, "split_dim": d, "pp": pp.rank, "dtype": str(p.dtype)}
        tensors[f"model/{g}"] = _snapshot(p, background)
        for kind, t in state.get(name, {}).items():
            index[f"{kind}/{g}"] = {"shape": full, "split_dim": d, "pp": pp.rank, "dtype": str(t.dtype)}
            tensors[f"{kind}/{g}"] = _snapshot(t, background)
    writer = dp.rank == 0
    shard_file = os.path.join(path, f"shard_tp{tp.rank}_pp{pp.rank}.pt")
    # Every cell's index (tp0 of each stage speaks for it) and who writes a shard.
    mine = {"writer": writer, "index": index if writer and tp.rank == 0 else None}
    gathered = [None] * (dist.get_world_size() if dist.is_initialized() else 1)
    if dist.is_initialized():
        dist.all_gather_object(gathered, mine)
    else:
        gathered = [mine]
    if not background:
        if writer:
            _write_shard(tensors, shard_file)
        if rank == 0:
            _write_manifest(path, gathered, step, seed, opt_step, config, tp, pp, dp, extra)
        if dist.is_initialized():
            dist.barrier()
        if rank == 0:
            with open(os.path.join(path, "COMPLETE"), "w") as f:
                f.write("ok\n")
        if dist.is_initialized():
            dist.barrier()
        return path

    writers = [r for r, part in enumerate(gathered) if part and part["writer"]]
    store = dist.distributed_c10d._get_default_store() if dist.is_initialized() else None
    key = f"dst/ckpt/{os.path.abspath(path)}"
    handle = PendingSave(path)

    def work():
        try:
            if writer:
                _write_shard(tensors, shard_file)
            if store is not None:
                store.set(f"{key}/{rank}", "ok")
            if rank == 0:
                _write_manifest(path, gathered, step, seed, opt_step, config, tp, pp, dp, extra)
                if store is not None:
                    store.wait([f"{key}/{r}" for r in writers], datetime.timedelta(seconds=timeout_s))
                with open(os.path.join(path, "COMPLETE"), "w") as f:
                    f.write("ok\n")
        except BaseException as e:  # noqa: BLE001 - surfaced by wait()
            handle.error = e

    t = threading.Thread(target=work, name=f"dst-ckpt-{step}", daemon=False)
    handle._thread = t
    t.start()
    return handle


def prune(root: str, keep: int) -> List[str]:
    """Delete all but the newest ``keep`` COMPLETE checkpoints under ``root``,
    and incomplete directories older than the newest complete one (writes
    that failed). Directories newer than it are left alone: a background
    write may still be filling one. Call from one process (rank 0) after a
    checkpoint is complete; returns the deleted paths."""
    if keep < 1 or not os.path.isdir(root):
        return []
    dirs = sorted(d for d in os.listdir(root) if d.startswith("step_") and os.path.isdir(os.path.join(root, d)))
    complete = [d for d in dirs if os.path.exists(os.path.join(root, d, "COMPLETE"))]
    if not complete:
        return []
    newest = complete[-1]
    doomed = complete[:-keep] + [d for d in dirs if d < newest and d not in complete]
    removed = []
    for d in sorted(doomed):
        shutil.rmtree(os.path.join(root, d), ignore_errors=True)
        removed.append(os.path.join(root, d))
    return removed


def latest(root: str) -> Optional[str]:
    """The newest COMPLETE checkpoint directory under ``root`` (or None)."""
    if not os.path.isdir(root):
        return None
    steps = sorted(d for d in os.listdir(root) if d.startswith("step_") and os.path.exists(os.path.join(root, d, "COMPLETE")))
    return os.path.join(root, steps[-1]) if steps else None


class _Reader:
    """Loads global tensors from a checkpoint written at any topology."""

    def __init__(self, path: str):
        self.path = path
        with open(os.path.join(path, "manifest.json")) as f:
            self.manifest = json.load(f)
        self.topo = self.manifest["topology"]
        self._cache: Dict[str, dict] = {}

    def _file(self, t: int, p: int) -> dict:
        key = f"shard_tp{t}_pp{p}.pt"
        if key not in self._cache:
            f = os.path.join(self.path, key)
            if not verify_shard(f):
                raise RuntimeError(f"checkpoint shard {f} does not match its recorded SHA-256")
            self._cache[key] = torch.load(f, map_location="cpu", weights_only=True)
        return self._cache[key]

    def full(self, key: str) -> Optional[torch.Tensor]:
        meta = self.manifest["tensors"].get(key)
        if meta is None:
            return None
        if meta["split_dim"] is None:
            return self._file(0, meta["pp"])[key]
        parts = [self._file(t, meta["pp"])[key] for t in range(self.topo["tp"])]
        return torch.cat(parts, dim=meta["split_dim"])


def load(path: str, model: nn.Module, opt, tp) -> dict:
    """Load weights (and optimizer state when present) into this rank's
    model/optimizer, resharding as needed. Returns the manifest."""
    from ..optim.fused_dp import FusedDPAdam
    from ..optim.precision import MasterWeightOptimizer

    rd = _Reader(path)
    params = list(model.named_parameters())
    masters = {}
    if isinstance(opt, MasterWeightOptimizer):
        masters = dict(zip([id(p) for p in opt.model_params], opt.master_params))

    def local(key, name, like):
        full = rd.full(key)
        if full is None:
            return None
        d = split_dim(model, name)
        if d is not None:
            n = like.shape[d]
            full = full.narrow(d, tp.rank * n, n)
        return full

    opt_step = float(rd.manifest.get("optimizer_step", 0.0))
    with torch.no_grad():
        for name, p in params:
            g = _global_name(model, name)
            w = local(f"model/{g}", name, p)
            if w is None:
                raise KeyError(f"checkpoint {path} has no tensor for {g}")
            p.copy_(w.to(p.dtype))
            if isinstance(opt, FusedDPAdam):
                src = local(f"master/{g}", name, p)
                ea, eas = local(f"exp_avg/{g}", name, p), local(f"exp_avg_sq/{g}", name, p)
                zeros = torch.zeros(p.shape)
                opt.load_full_state(
                    p,
                    src if src is not None else w.float(),
                    ea if ea is not None else zeros,
                    eas if eas is not None else zeros,
                    int(opt_step),
                )
            elif isinstance(opt, MasterWeightOptimizer) and id(p) in masters:
                m = masters[id(p)]
                src = local(f"master/{g}", name, p)
                m.copy_(src if src is not None else w.float())
                ea, eas = local(f"exp_avg/{g}", name, p), local(f"exp_avg_sq/{g}", name, p)
                if ea is not None and eas is not None:
                    st = opt._state(m)
                    st["exp_avg"].copy_(ea)
                    st["exp_avg_sq"].copy_(eas)
                    st["step"] = torch.tensor(opt_step)
            elif isinstance(opt, torch.optim.Optimizer):
                ea, eas = local(f"exp_avg/{g}", name, p), local(f"exp_avg_sq/{g}", name, p)
                if ea is not None and eas is not None:
                    fused = bool(opt.defaults.get("fused"))  # fused Adam keeps its step on the params' device
                    opt.state[p] = {
                        "step": torch.tensor(float(opt_step), dtype=torch.float32,
                                             device=p.device if fused else "cpu"),
                        "exp_avg": ea.to(p.device, p.dtype).clone(),
                        "exp_avg_sq": eas.to(p.device, p.dtype).clone(),
                    }
    return rd.manifest


def inspect(path: str) -> dict:
    """Summary of a checkpoint directory: step, topology, tensor count and
    bytes, and which shards are missing or fail their checksum."""
    with open(os.path.join(path, "manifest.json")) as f:
        man = json.load(f)
    topo = man["topology"]
    missing, corrupt, nbytes = [], [], 0
    for t in range(topo["tp"]):
        for p in range(topo["pp"]):
            f = os.path.join(path, f"shard_tp{t}_pp{p}.pt")
            if not os.path.exists(f):
                missing.append(os.path.basename(f))
                continue
            nbytes += os.path.getsize(f)
            if not verify_shard(f):
                corrupt.append(os.path.basename(f))
    return {
        "path": path,
        "step": man["step"],
        "complete": os.path.exists(os.path.join(path, "COMPLETE")),
        "topology": topo,
        "tensors": len(man["tensors"]),
        "bytes": nbytes,
        "missing": missing,
        "corrupt": corrupt,
        "ok": not missing and not corrupt and os.path.exists(os.path.join(path, "COMPLETE")),
    }


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="inspect / verify a sharded checkpoint")
    ap.add_argument("path", help="a step_XXXXXXXX directory, or a root (its latest complete checkpoint)")
    a = ap.parse_args(argv)
    path = a.path
    if not os.path.exists(os.path.join(path, "manifest.json")):
        path = latest(path) or path
    info = inspect(path)
    print(json.dumps(info, indent=1))
    raise SystemExit(0 if info["ok"] else 1)


if __name__ == "__main__":
    main()
