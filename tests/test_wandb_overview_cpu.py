"""W&B overview view: layout from the run config, naming, equality check and
creation through a stand-in for the optional wandb-workspaces package."""

import sys
import types

from wavelet_b200 import wandb_overview as wo


def test_inputs_and_sections():
    assert wo.overview_inputs({"trainer": {}}) == ("sft", [], [])
    cfg = {"orchestrator": {"envs": [{"id": "equation_builder@1.0"}, {"name": "polaris", "id": "x"}],
                            "verifier_env_id": None},
           "eval": {"env": [{"id": "aime@2"}]}}
    flavor, tr, ev = wo.overview_inputs(cfg)
    assert (flavor, tr, ev) == ("rl", ["equation_builder", "polaris"], ["aime"])
    secs = wo.overview_sections(flavor, tr, ev)
    assert [s["name"] for s in secs] == ["train", "eval", "stability", "inference", "performance", "resources"]
    assert secs[0]["regexes"] == [r"train/(equation_builder|polaris)/.*"]
    assert secs[1]["regexes"][0].startswith("eval/(aime)/")
    assert wo.overview_sections("rl", ["only"])[0]["name"] == "train/only"
    assert wo.overview_sections("sft")[0]["metrics"][0] == "loss"


def test_view_names():
    assert wo.next_view_name("overview", []) == "overview"
    assert wo.next_view_name("overview", ["overview"]) == "overview-v2"
    assert wo.next_view_name("overview", ["overview", "overview-v2", "overview-v7"]) == "overview-v8"


def _fake_workspaces(saved):
    class Obj:
        def __init__(self, **kw):
            self.__dict__.update(kw)

    class LinePlot(Obj):
        def __init__(self, x, y=None, metric_regex=None):
            super().__init__(x=x, y=y, metric_regex=metric_regex)

    class Workspace(Obj):
        existing = {}

        @classmethod
        def from_url(cls, url):
            return cls.existing[url.rsplit("=", 1)[1]]

        def save(self):
            saved.append(self)
            self.url = f"https://wandb.ai/{self.entity}/{self.project}?nw={self.name}"

    reports = types.ModuleType("wandb_workspaces.reports.v2")
    reports.LinePlot = LinePlot
    wsmod = types.ModuleType("wandb_workspaces.workspaces")
    wsmod.Workspace = Workspace
    wsmod.Section = Obj
    wsmod.SectionLayoutSettings = Obj
    wsmod.WorkspaceSettings = Obj
    root = types.ModuleType("wandb_workspaces")
    rep = types.ModuleType("wandb_workspaces.reports")
    return {"wandb_workspaces": root, "wandb_workspaces.reports": rep, "wandb_workspaces.reports.v2": reports,
            "wandb_workspaces.workspaces": wsmod}, Workspace


def test_ensure_creates_once(monkeypatch):
    saved = []
    mods, Workspace = _fake_workspaces(saved)
    for k, v in mods.items():
        monkeypatch.setitem(sys.modules, k, v)
    url = wo.ensure_overview_view("ent", "proj", "sft", lister=lambda e, p: [("other", "nw-a")])
    assert url.endswith("nw=overview") and len(saved) == 1
    # an existing view with the same panels -> nothing new
    Workspace.existing["b"] = saved[0]
    assert wo.ensure_overview_view("ent", "proj", "sft", lister=lambda e, p: [("overview", "nw-b-v")]) is None
    # a different layout (RL) under the same base name -> versioned name
    url = wo.ensure_overview_view("ent", "proj", "rl", ["env"], lister=lambda e, p: [("overview", "nw-b-v")])
    assert url.endswith("nw=overview-v2") and len(saved) == 2


def test_missing_package_is_not_fatal(monkeypatch):
    monkeypatch.setitem(sys.modules, "wandb_workspaces", None)
    run = types.SimpleNamespace(entity="e", project="p")
    cfg = types.SimpleNamespace(mode="online", create_overview=True)
    assert wo.maybe_create_overview(run, {}, cfg) is None
    assert wo.maybe_create_overview(run, {}, types.SimpleNamespace(mode="offline", create_overview=True)) is None
