"""Custom algorithm definitions loaded by tests/test_algorithms_cpu.py."""

from dataclasses import dataclass, replace

from wavelet_b200.data.rl import RLExample
from wavelet_b200.orchestrator.algorithms import BaseAlgorithm, register_algorithm


@register_algorithm("scale")
@dataclass(frozen=True)
class ScaleRewards(BaseAlgorithm):
    factor: float

    def score_group(self, records):
        return [replace(r, advantage=float(r.reward or 0.0) * self.factor) for r in records]


@register_algorithm("rollout_only")
class RolloutOnly:  # no score_group
    def score_rollout(self, record):
        return record


class PlainAlgorithm(BaseAlgorithm):  # found by its attribute name
    pass


NOT_A_FACTORY = 7


@register_algorithm("twice")
class TwiceA(BaseAlgorithm):
    pass


@register_algorithm("twice")
class TwiceB(BaseAlgorithm):
    pass


@register_algorithm("bad_rollout")
class BadRollout(BaseAlgorithm):
    def score_rollout(self, record):
        return {"record": record}


@register_algorithm("drops_one")
class DropsOne(BaseAlgorithm):
    def score_group(self, records):
        return records[:-1]


@register_algorithm("both")
class Both(BaseAlgorithm):
    def score_rollout(self, record):
        return replace(record, advantage=float(record.reward or 0.0))

    def score_group(self, records):
        return [replace(r, advantage=float(r.advantage or 0.0) + 1.0) for r in records]


@register_algorithm("offset")
def make_offset(*, offset: float):
    class Offset(BaseAlgorithm):
        def score_rollout(self, record: RLExample) -> RLExample:
            return replace(record, advantage=float(record.reward or 0.0) + offset)

    return Offset()
