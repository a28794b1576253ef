"""Checkpoint / resume.

The reference has no checkpoint code; its design names
``PolicyEngine::SaveCheckpoint/LoadCheckpoint(path)`` writing
``{checkpoint_dir}/step_{N}`` every ``checkpoint_interval`` and persists
configuration as ``key=value`` text (turbol_vllm/src/core/config.cpp:19-59).
This module defines the format:

    <dir>/step_<N>/
        policy.pt                 model weights (``policy_tp<t>_pp<p>.pt`` per
                                  tensor/pipeline-parallel rank when sharded)
        optim.pt                  optimizer state (``optim_dp<d>...`` when the
                                  state is sharded across data-parallel ranks)
        trainer.pt                everything else the trainer needs to continue
                                  bit-identically (counters, env state, RNG)
        replay.pt                 optional replay-buffer contents
        config.cfg                configuration, ``key=value`` (readable by
                                  ``turbol_b200.Config.load``)
        COMPLETE<sfx>             written last by each saving rank, with the
                                  layout of the save (tp, pp and dp sizes).  A
                                  step counts as complete only when the marker
                                  of every rank of that layout is present; an
                                  interrupted or partial save is ignored by
                                  ``latest_step`` and refused by ``load_checkpoint``.

File suffixes: ``_tp<t>_pp<p>`` when the layout has more than one tensor- or
pipeline-parallel rank (the model is sharded), and ``_dp<d>`` on the files of
state that differs between data-parallel ranks (sharded optimizer moments,
each rank's environments and RNG).  The policy of a (tp, pp) shard is written
once, by data-parallel rank 0.  A trainer reports its place in the layout with
``checkpoint_ranks()`` (``tp_rank``, ``pp_rank``, ``dp_rank``, ``layout``);
explicit arguments override it.

A trainer participates through ``state_dict()`` returning a dict whose
``"policy"`` and ``"optim"`` entries go to their own files and whose other
entries go to ``trainer.pt``, and ``load_state_dict(d)`` taking the same dict.

Saves can run in the background: tensors are snapshotted to host memory on the
calling thread (so training may continue and modify them), then a worker
thread writes the files.
"""
from __future__ import annotations

import json
import os
import re
import shutil
import threading
from dataclasses import asdict, is_dataclass
from typing import Any, Dict, Optional

import torch

_STEP_RE = re.compile(r"^step_(\d+)$")


def _to_host(obj):
    """Deep copy with every tensor moved to host memory (detached)."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _to_host(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_host(v) for v in obj)
    return obj


def _flatten_config(cfg, prefix="") -> Dict[str, str]:
    if cfg is None:
        return {}
    if is_dataclass(cfg):
        cfg = asdict(cfg)
    out = {}
    for k, v in dict(cfg).items():
        key = f"{prefix}{k}"
        if isinstance(v, dict) or is_dataclass(v):
            out.update(_flatten_config(v, key + "."))
        elif isinstance(v, (list, tuple)):
            out[key] = ",".join(str(x) for x in v)
        else:
            out[key] = str(v)
    return out


def _write_config(path: str, cfg) -> None:
    flat = _flatten_config(cfg)
    try:
        from .._native import core

        c = core().Config()
        for k, v in flat.items():
            c.set(k, v)
        st = c.save(path)
        if st.ok():
            return
    except (ImportError, AttributeError):
        pass
    with open(path, "w") as f:  # same format, without the native core
        f.write("# turbol_b200 checkpoint configuration\n")
        for k in sorted(flat):
            f.write(f"{k}={flat[k]}\n")


def read_config(path: str) -> Dict[str, str]:
    out = {}
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line or line.startswith("#") or "=" not in line:
                continue
            k, v = line.split("=", 1)
            out[k.strip()] = v.strip()
    return out


def _suffix(tp: int, pp: int, dp: Optional[int], sharded: bool) -> str:
    s = ""
    if dp is not None:
        s += f"_dp{dp}"
    if sharded:
        s += f"_tp{tp}_pp{pp}"
    return s


def _resolve_ranks(trainer, tp_rank, pp_rank, dp_rank, layout):
    """Fills unset rank arguments from ``trainer.checkpoint_ranks()``."""
    auto = {}
    if trainer is not None and hasattr(trainer, "checkpoint_ranks"):
        auto = trainer.checkpoint_ranks() or {}
    tp_rank = auto.get("tp_rank", 0) if tp_rank is None else tp_rank
    pp_rank = auto.get("pp_rank", 0) if pp_rank is None else pp_rank
    if dp_rank is None:
        dp_rank = auto.get("dp_rank")
    lay = dict(auto.get("layout") or {})
    lay.update(layout or {})
    tp = int(lay.get("tp", max(1, tp_rank + 1)))
    pp = int(lay.get("pp", max(1, pp_rank + 1)))
    dp = int(lay.get("dp", 0 if dp_rank is None else dp_rank + 1))
    if dp_rank is not None and dp < 1:
        raise ValueError("a per-data-parallel-rank save needs layout['dp'] >= 1")
    return int(tp_rank), int(pp_rank), dp_rank, {"tp": tp, "pp": pp, "dp": dp if dp_rank is not None else 0}


def _marker_names(layout) -> set:
    sharded = layout["tp"] * layout["pp"] > 1
    dps = [None] if layout["dp"] == 0 else list(range(layout["dp"]))
    return {f"COMPLETE{_suffix(t, p, d, sharded)}" for t in range(layout["tp"]) for p in range(layout["pp"])
            for d in dps}


def _read_marker(path: str):
    try:
        with open(path) as f:
            text = f.read().strip()
        d = json.loads(text)
        if isinstance(d, dict) and {"tp", "pp", "dp"} <= set(d):
            return {"tp": int(d["tp"]), "pp": int(d["pp"]), "dp": int(d["dp"])}
    except (OSError, ValueError):
        pass
    return None


def step_complete(path: str) -> bool:
    """True when every rank of the save's layout wrote its marker in ``path``."""
    if not os.path.isdir(path):
        return False
    names = {f for f in os.listdir(path) if f.startswith("COMPLETE")}
    if not names:
        return False
    for n in sorted(names):
        lay = _read_marker(os.path.join(path, n))
        if lay is None:
            if n == "COMPLETE":  # a single-process save of the first format
                return True
            continue
        return _marker_names(lay) <= names
    return False


class SaveHandle:
    def __init__(self, path: str, thread: Optional[threading.Thread]):
        self.path = path
        self._thread = thread
        self.error: Optional[BaseException] = None

    def wait(self) -> str:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self.error is not None:
            raise self.error
        return self.path

    def done(self) -> bool:
        return self._thread is None or not self._thread.is_alive()


def save_checkpoint(directory: str, step: int, trainer=None, *, state: Optional[Dict[str, Any]] = None,
                    config=None, replay: Optional[Dict[str, Any]] = None, tp_rank: Optional[int] = None,
                    pp_rank: Optional[int] = None, dp_rank: Optional[int] = None, layout: Optional[dict] = None,
                    write_config: bool = True, background: bool = False,
                    keep_last: Optional[int] = None) -> SaveHandle:
    """Writes this rank's files of ``<directory>/step_<step>/``.  Every rank of
    a parallel job calls it (each writes its own shards and marker).
    ``state`` defaults to ``trainer.state_dict()``; ``config`` to
    ``trainer.cfg``; the ranks and ``layout`` ({"tp", "pp", "dp"} sizes) to
    ``trainer.checkpoint_ranks()``.  With ``background=True`` returns at once
    after the host snapshot; call ``.wait()`` on the handle before relying on
    the files.  ``keep_last`` (applied by the lead rank) deletes all but the
    newest ``keep_last`` complete steps; an incomplete newer step that other
    ranks may still be writing is never counted or touched."""
    tp_rank, pp_rank, dp_rank, lay = _resolve_ranks(trainer, tp_rank, pp_rank, dp_rank, layout)
    lead = tp_rank == 0 and pp_rank == 0 and not dp_rank
    if state is None:
        if trainer is None:
            raise ValueError("save_checkpoint needs a trainer or a state dict")
        state = trainer.state_dict()
    if config is None and trainer is not None:
        config = getattr(trainer, "cfg", None)
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    snap = _to_host(dict(state))
    rep = _to_host(replay) if replay is not None else None
    path = os.path.join(directory, f"step_{int(step)}")
    sharded = lay["tp"] * lay["pp"] > 1
    sfx = _suffix(tp_rank, pp_rank, None, sharded)
    osfx = _suffix(tp_rank, pp_rank, dp_rank, sharded)
    marker = json.dumps({"step": int(step), **lay})

    def write():
        os.makedirs(path, exist_ok=True)
        policy = snap.pop("policy", None)
        optim = snap.pop("optim", None)
        if policy is not None and (dp_rank is None or dp_rank == 0):
            torch.save(policy, os.path.join(path, f"policy{sfx}.pt"))
        if optim is not None:
            torch.save(optim, os.path.join(path, f"optim{osfx}.pt"))
        torch.save(snap, os.path.join(path, f"trainer{osfx}.pt"))
        if rep is not None:
            torch.save(rep, os.path.join(path, f"replay{osfx}.pt"))
        if write_config and config is not None and lead:
            _write_config(os.path.join(path, "config.cfg"), config)
        tmp = os.path.join(path, f".COMPLETE{osfx}.tmp")
        with open(tmp, "w") as f:
            f.write(marker + "\n")
        os.replace(tmp, os.path.join(path, f"COMPLETE{osfx}"))
        if keep_last is not None and lead:
            for old in list_steps(directory)[:-keep_last]:
                if old < int(step):
                    shutil.rmtree(os.path.join(directory, f"step_{old}"), ignore_errors=True)

    if not background:
        write()
        return SaveHandle(path, None)
    handle = SaveHandle(path, None)

    def run():
        try:
            write()
        except BaseException as e:  # surfaced by wait()
            handle.error = e

    t = threading.Thread(target=run, name=f"turbol-ckpt-{step}", daemon=False)
    handle._thread = t
    t.start()
    return handle


def list_steps(directory: str):
    """Completed checkpoint steps in ``directory``, ascending."""
    if not os.path.isdir(directory):
        return []
    steps = []
    for name in os.listdir(directory):
        m = _STEP_RE.match(name)
        if not m:
            continue
        if step_complete(os.path.join(directory, name)):
            steps.append(int(m.group(1)))
    return sorted(steps)


def latest_step(directory: str) -> Optional[int]:
    s = list_steps(directory)
    return s[-1] if s else None


def load_checkpoint(directory: str, step: Optional[int] = None, trainer=None, *, map_location="cpu",
                    tp_rank: Optional[int] = None, pp_rank: Optional[int] = None, dp_rank: Optional[int] = None,
                    layout: Optional[dict] = None, config=None, strict_config: bool = True) -> Dict[str, Any]:
    """Reads this rank's files of ``<directory>/step_<step>`` (the latest
    complete one by default) and returns the state dict (``policy``, ``optim``
    and the trainer entries, plus ``replay`` and ``config`` when present).
    With ``trainer`` the state is also loaded into it, and the ranks default
    to ``trainer.checkpoint_ranks()``.  The step must be complete for its
    layout and must hold this rank's marker.  With ``config`` (or
    ``trainer.cfg``) the saved configuration must match key for key unless
    ``strict_config=False``."""
    tp_rank, pp_rank, dp_rank, lay = _resolve_ranks(trainer, tp_rank, pp_rank, dp_rank, layout)
    if step is None:
        step = latest_step(directory)
        if step is None:
            raise FileNotFoundError(f"no completed checkpoint under {directory}")
    path = os.path.join(directory, f"step_{int(step)}")
    sharded = lay["tp"] * lay["pp"] > 1
    sfx = _suffix(tp_rank, pp_rank, None, sharded)
    osfx = _suffix(tp_rank, pp_rank, dp_rank, sharded)
    if not step_complete(path):
        raise FileNotFoundError(f"{path} is not a complete checkpoint (a rank's marker is missing)")
    own = os.path.join(path, f"COMPLETE{osfx}")
    if not os.path.exists(own) and not (osfx == "" and os.path.exists(os.path.join(path, "COMPLETE"))):
        raise FileNotFoundError(f"{path} has no files of this rank (marker COMPLETE{osfx} missing)")
    saved_lay = _read_marker(own)
    if saved_lay is not None and saved_lay != lay:
        raise ValueError(f"checkpoint layout {saved_lay} differs from this job's {lay}")
    state: Dict[str, Any] = torch.load(os.path.join(path, f"trainer{osfx}.pt"), map_location=map_location,
                                       weights_only=False)
    pol = os.path.join(path, f"policy{sfx}.pt")
    if os.path.exists(pol):
        state["policy"] = torch.load(pol, map_location=map_location, weights_only=False)
    opt = os.path.join(path, f"optim{osfx}.pt")
    if os.path.exists(opt):
        state["optim"] = torch.load(opt, map_location=map_location, weights_only=False)
    rep = os.path.join(path, f"replay{osfx}.pt")
    if os.path.exists(rep):
        state["replay"] = torch.load(rep, map_location=map_location, weights_only=False)
    cfg_path = os.path.join(path, "config.cfg")
    if os.path.exists(cfg_path):
        saved_cfg = read_config(cfg_path)
        state["config"] = saved_cfg
        want = config if config is not None else (getattr(trainer, "cfg", None) if trainer is not None else None)
        if want is not None and strict_config:
            cur = _flatten_config(want)
            diff = {k for k in set(cur) | set(saved_cfg) if cur.get(k) != saved_cfg.get(k)}
            if diff:
                raise ValueError(f"checkpoint configuration differs in {sorted(diff)}")
    state["step"] = int(step)
    if trainer is not None:
        trainer.load_state_dict({k: v for k, v in state.items() if k not in ("replay", "config", "step")})
    return state


__all__ = ["save_checkpoint", "load_checkpoint", "latest_step", "list_steps", "read_config", "SaveHandle",
           "step_complete"]
