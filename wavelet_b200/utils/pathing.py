"""Run-directory layout.

    <output_dir>/configs/attempt_<n>/resolved/   resolved role configs of launch n
    <output_dir>/configs/latest -> attempt_<n>
    <output_dir>/logs/attempt_<n>/               role logs of launch n (logs/latest)
    <output_dir>/checkpoint-<step>/STABLE        committed checkpoint
    <output_dir>/rollouts/step-XXXXXX/           rollout queue (transport.queue)
    <output_dir>/policies/step-XXXXXX/           policy snapshots (transport.policy)

Same names as the reference (utils/pathing.py:58-217) so tools interoperate.
"""

from __future__ import annotations

import os
import shlex
import shutil
from collections.abc import Iterable
from dataclasses import dataclass
from pathlib import Path

STABLE = "STABLE"
RUN_STATE_ENTRIES = (
    "configs", "eval_metrics.jsonl", "evals", "events", "events.jsonl", "heartbeat.json", "logs",
    "metrics.csv", "metrics.jsonl", "policies", "rollouts", "run_metadata.json", "wandb",
)


@dataclass(frozen=True)
class LaunchAttempt:
    config_attempt_dir: Path
    config_dir: Path
    log_dir: Path


def _attempts(root: Path) -> set[int]:
    out = set()
    for p in root.glob("attempt_*"):
        s = p.name[len("attempt_"):]
        if p.is_dir() and s.isdigit():
            out.add(int(s))
    return out


def _repoint_latest(root: Path, target: Path) -> None:
    tmp = root / f".latest-{os.getpid()}"
    if tmp.is_symlink() or tmp.exists():
        tmp.unlink()
    tmp.symlink_to(target.name, target_is_directory=True)
    os.replace(tmp, root / "latest")


def create_launch_attempt(output_dir: Path) -> LaunchAttempt:
    cfg_root = Path(output_dir) / "configs"
    log_root = Path(output_dir) / "logs"
    cfg_root.mkdir(parents=True, exist_ok=True)
    log_root.mkdir(parents=True, exist_ok=True)
    n = max(_attempts(cfg_root) | _attempts(log_root), default=0) + 1
    a = cfg_root / f"attempt_{n}"
    resolved = a / "resolved"
    logs = log_root / f"attempt_{n}"
    resolved.mkdir(parents=True)
    logs.mkdir()
    _repoint_latest(cfg_root, a)
    _repoint_latest(log_root, logs)
    return LaunchAttempt(a, resolved, logs)


def config_paths_in_argv(argv: list[str]) -> list[Path]:
    out, i = [], 0
    while i < len(argv):
        t = argv[i]
        if t == "@" and i + 1 < len(argv):
            out.append(Path(argv[i + 1]))
            i += 2
            continue
        if t.startswith("@") and len(t) > 1:
            out.append(Path(t[1:]))
        i += 1
    return out


def write_launch_artifacts(attempt: LaunchAttempt, *, command: str, argv: list[str]) -> None:
    (attempt.config_attempt_dir / "command.txt").write_text(shlex.join(["wavelet", command, *argv]) + "\n")
    srcs = config_paths_in_argv(argv)
    for i, s in enumerate(srcs, 1):
        if s.is_file():
            stem = command if len(srcs) == 1 else f"{command}_{i}"
            dst = attempt.config_attempt_dir / f"{stem}{s.suffix or '.yaml'}"
            if s.resolve() != dst.resolve():
                shutil.copyfile(s, dst)


def get_config_dir(output_dir: Path) -> Path:
    latest = Path(output_dir) / "configs" / "latest" / "resolved"
    return latest if latest.exists() else Path(output_dir) / "configs"


def checkpoint_dir(output_dir: Path, step: int) -> Path:
    return Path(output_dir) / f"checkpoint-{step}"


def is_stable(path: Path) -> bool:
    return path.is_dir() and (path / STABLE).exists()


def list_checkpoint_steps(output_dir: Path, stable_only: bool = True) -> list[int]:
    root = Path(output_dir)
    if not root.exists():
        return []
    steps = []
    for p in root.glob("checkpoint-*"):
        s = p.name[len("checkpoint-"):]
        if s.isdigit() and (not stable_only or is_stable(p)):
            steps.append(int(s))
    return sorted(steps)


def latest_checkpoint_step(output_dir: Path) -> int | None:
    steps = list_checkpoint_steps(output_dir)
    return steps[-1] if steps else None


def resolve_resume_dir(output_dir: Path, resume_step: int | None, resume_dir: Path | None) -> Path | None:
    """-1 means the latest stable checkpoint; None means no resume."""
    if resume_dir is not None:
        if not is_stable(resume_dir):
            raise FileNotFoundError(f"checkpoint {resume_dir} is missing or not STABLE")
        return resume_dir
    if resume_step is None:
        return None
    if resume_step == -1:
        s = latest_checkpoint_step(output_dir)
        if s is None:
            raise FileNotFoundError(f"no stable checkpoint under {output_dir}")
        return checkpoint_dir(output_dir, s)
    p = checkpoint_dir(output_dir, resume_step)
    if not is_stable(p):
        raise FileNotFoundError(f"checkpoint {p} is missing or not STABLE")
    return p


def existing_run_state_entries(output_dir: Path) -> list[str]:
    root = Path(output_dir)
    if not root.exists():
        return []
    out = [n for n in RUN_STATE_ENTRIES if (root / n).exists() or (root / n).is_symlink()]
    return out + sorted(p.name for p in root.glob("checkpoint-*"))


def has_run_state(output_dir: Path) -> bool:
    return bool(existing_run_state_entries(output_dir))


def _refuse_unsafe_root(root: Path) -> None:
    """Directories that are clearly not run directories are never cleaned."""
    reasons = []
    if root == Path(root.anchor):
        reasons.append("the filesystem root")
    if root == Path.home().absolute():
        reasons.append("the home directory")
    cwd = Path.cwd().absolute()
    if cwd == root or cwd.is_relative_to(root):
        reasons.append("the current working directory or one of its parents")
    if reasons:
        raise ValueError(f"clean_output_dir=true refuses to clean '{root}': it is " + " and ".join(reasons)
                         + ". Point output_dir at a dedicated run directory.")


def clean_output_dir(output_dir: Path) -> None:
    """Remove the run state; the directory itself goes too when nothing else
    (unrelated files) is left in it."""
    root = Path(output_dir)
    if not root.exists():
        return
    for n in RUN_STATE_ENTRIES:
        p = root / n
        if p.is_symlink() or p.is_file():
            p.unlink()
        elif p.is_dir():
            shutil.rmtree(p)
    for p in root.glob("checkpoint-*"):
        if p.is_dir():
            shutil.rmtree(p)
    if root.is_dir() and not any(root.iterdir()):
        root.rmdir()


def validate_output_dir(output_dir: Path, *, clean: bool, resuming: bool,
                        protected_paths: Iterable[Path | str | None] = ()) -> None:
    """Refuse to overwrite a previous run unless resuming or cleaning
    (reference utils/pathing.py:186-259): cleaning and resuming exclude each
    other, cleaning never touches the filesystem root, the home or working
    directory, nor an input (model, adapter) that lies inside the run."""
    if clean and resuming:
        raise ValueError("clean_output_dir=true cannot be used with checkpoint resume. "
                         "Choose either a clean run or an explicit resume.")
    if resuming:
        return
    root = Path(output_dir).absolute()
    if clean:
        _refuse_unsafe_root(root)
        inside = [str(p) for p in protected_paths
                  if p is not None and Path(p).exists() and Path(p).absolute().is_relative_to(root)]
        if inside:
            raise ValueError("clean_output_dir=true would remove required input path(s): " + ", ".join(inside))
        clean_output_dir(output_dir)
        return
    entries = existing_run_state_entries(output_dir)
    if entries:
        preview = ", ".join(entries[:5]) + (", ..." if len(entries) > 5 else "")
        raise FileExistsError(
            f"{output_dir} already contains run state ({preview}); use a fresh output_dir, set "
            "clean_output_dir=true, or resume from a checkpoint"
        )
