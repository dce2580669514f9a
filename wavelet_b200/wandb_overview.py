"""Curated W&B workspace view ("overview") for a run (reference
wandb_overview.py).

The layout is plain data (``overview_sections``): sections of line plots
keyed by this framework's metric names: train (SFT loss / progress, or RL
reward / advantage / sample fate, per environment when there are several),
eval (avg@k / pass@k per eval environment), stability, inference (wall-clock
x axis), performance and resources.  ``ensure_overview_view`` turns it into a
workspace with the ``wandb-workspaces`` package (imported only there; it is
optional and not bundled), unless the project already holds an overview with
the same panels; new views are named ``overview``, ``overview-v2``, ...
"""

from __future__ import annotations

import logging
import re
from collections.abc import Mapping, Sequence
from typing import Any

log = logging.getLogger("wavelet")

VIEW_BASE = "overview"
GRID = (4, 6)  # columns, rows per section

SFT_TRAIN = ("loss", "train/loss", "val/loss", "progress/epoch", "progress/total_samples", "progress/total_tokens")
RL_TRAIN = ("reward/all/mean", "advantage/all/mean", "progress/samples", "progress/tokens", "fate/all/trainable",
            "fate/all/filtered", "fate/all/errored")
STABILITY = ("optim/grad_norm", "entropy/mean", "kl/mismatch", "lr")
PERFORMANCE = ("perf/mfu", "perf/tokens_per_second", "perf/train_tokens_per_second", "time/step",
               "time/forward_backward", "time/wait_for_batch")
RESOURCES = ("cuda_memory_allocated_bytes", "cuda_memory_reserved_bytes", "disk_free_ratio",
             "checkpoint_disk_free_ratio")


def _sec(name: str, metrics: Sequence[str] = (), regexes: Sequence[str] = (), x: str = "step") -> dict:
    return {"name": name, "x": x, "metrics": list(metrics), "regexes": list(regexes)}


def overview_sections(flavor: str, train_envs: Sequence[str] = (), eval_envs: Sequence[str] = ()) -> list[dict]:
    if flavor == "sft":
        train = _sec("train", SFT_TRAIN)
    else:
        several = len(train_envs) > 1
        train = _sec(f"train/{train_envs[0]}" if len(train_envs) == 1 else "train", RL_TRAIN,
                     [rf"train/({'|'.join(map(re.escape, train_envs))})/.*"] if several else [])
    envs = "|".join(map(re.escape, eval_envs)) or ".*"
    return [train,
            _sec("eval", regexes=[rf"eval/({envs})/(avg@.*|pass@.*|pass\^.*|failed_rollouts)"]),
            _sec("stability", STABILITY),
            _sec("inference", regexes=[r"inference/.*"], x="RelativeTime(Wall)"),
            _sec("performance", PERFORMANCE),
            _sec("resources", RESOURCES)]


def _names(envs: Any) -> list[str]:
    out = []
    for e in envs if isinstance(envs, list) else []:
        if isinstance(e, Mapping):
            n = e.get("name") or e.get("id")
            if isinstance(n, str) and n:
                out.append(n.split("@", 1)[0])
    return out


def overview_inputs(run_config: Mapping[str, Any] | None) -> tuple[str, list[str], list[str]]:
    """(flavor, train environment names, eval environment names) of a
    serialised run config: RL when it has an orchestrator section."""
    if not run_config or "orchestrator" not in run_config:
        return "sft", [], []
    o = run_config.get("orchestrator")
    train = _names(o.get("envs")) if isinstance(o, Mapping) else []
    vid = o.get("verifier_env_id") if isinstance(o, Mapping) else None
    if isinstance(vid, str) and vid:
        train.append(vid.split("@", 1)[0])
    ev = run_config.get("eval")
    return "rl", train, _names(ev.get("env")) if isinstance(ev, Mapping) else []


def view_signature(sections: Sequence[dict]) -> tuple:
    """What makes two overviews equal: section names and their panels."""
    return tuple((s["name"], tuple((s["x"], (m,), None) for m in s["metrics"])
                  + tuple((s["x"], (), r) for r in s["regexes"])) for s in sections)


def next_view_name(base: str, existing: Sequence[str]) -> str:
    if base not in existing:
        return base
    nums = [int(n[len(base) + 2:]) for n in existing if n.startswith(base + "-v") and n[len(base) + 2:].isdigit()]
    return f"{base}-v{max(nums, default=1) + 1}"


def _workspace_sections(ws, wr, sections: Sequence[dict]) -> list:
    out = []
    for s in sections:
        panels = [wr.LinePlot(x=s["x"], y=[m]) for m in s["metrics"]] + [
            wr.LinePlot(x=s["x"], metric_regex=r) for r in s["regexes"]]
        out.append(ws.Section(name=s["name"], is_open=True, panels=panels,
                              layout_settings=ws.SectionLayoutSettings(columns=GRID[0], rows=GRID[1])))
    return out


def _signature_of_workspace(sections) -> tuple:
    return tuple((sec.name, tuple((getattr(p.x, "name", p.x), tuple(getattr(m, "name", m) for m in (p.y or ())),
                                   p.metric_regex) for p in sec.panels)) for sec in sections)


def list_views(entity: str, project: str) -> list[tuple[str, str]]:
    """(display name, internal name) of the project's saved views."""
    import wandb
    from wandb_workspaces.workspaces.internal import execute_graphql

    q = """query Views($entity: String!, $project: String!) { project(name: $project, entityName: $entity) {
           allViews(viewType: "project-view") { edges { node { name displayName } } } } }"""
    r = execute_graphql(wandb.Api(), q, {"entity": entity, "project": project})
    edges = ((r.get("project") or {}).get("allViews") or {}).get("edges") or []
    return [(e["node"]["displayName"], e["node"]["name"]) for e in edges
            if isinstance(e, Mapping) and isinstance(e.get("node"), Mapping)
            and isinstance(e["node"].get("displayName"), str) and isinstance(e["node"].get("name"), str)]


def ensure_overview_view(entity: str, project: str, flavor: str, train_envs: Sequence[str] = (),
                         eval_envs: Sequence[str] = (), lister=None) -> str | None:
    """Save a new overview view unless an equal one exists; returns its URL
    (None when nothing was created).  Needs ``wandb-workspaces``."""
    import wandb_workspaces.reports.v2 as wr
    import wandb_workspaces.workspaces as ws

    spec = overview_sections(flavor, train_envs, eval_envs)
    want = _signature_of_workspace(_workspace_sections(ws, wr, spec))
    views = [(d, n) for d, n in (lister or list_views)(entity, project)
             if d == VIEW_BASE or d.startswith(VIEW_BASE + "-v")]
    for _, internal in views:
        slug = internal.removeprefix("nw-").removesuffix("-v")
        try:
            have = ws.Workspace.from_url(f"https://wandb.ai/{entity}/{project}?nw={slug}")
        except Exception as e:  # an unreadable view does not block a new one
            log.warning("cannot read W&B view %s: %s", internal, e)
            continue
        if _signature_of_workspace(have.sections) == want:
            return None
    w = ws.Workspace(entity=entity, project=project, name=next_view_name(VIEW_BASE, [d for d, _ in views]),
                     sections=_workspace_sections(ws, wr, spec), auto_generate_panels=False,
                     settings=ws.WorkspaceSettings(x_axis="step"))
    w.save()
    return w.url


def maybe_create_overview(run: Any, run_config: Mapping | None, wandb_cfg: Any) -> str | None:
    """Called once after ``wandb.init`` of an online run with
    ``wandb.create_overview``; failures are logged, never raised."""
    if getattr(wandb_cfg, "mode", None) != "online" or not getattr(wandb_cfg, "create_overview", False):
        return None
    entity, project = getattr(run, "entity", None), getattr(run, "project", None)
    if not isinstance(entity, str) or not isinstance(project, str):
        log.warning("cannot create the W&B overview without entity and project")
        return None
    try:
        flavor, tr, ev = overview_inputs(run_config)
        url = ensure_overview_view(entity, project, flavor, tr, ev)
        if url:
            log.info("created W&B overview view: %s", url)
        return url
    except ImportError:
        log.warning("the W&B overview needs the wandb-workspaces package; skipped")
    except Exception:
        log.warning("failed to create the W&B overview view", exc_info=True)
    return None
