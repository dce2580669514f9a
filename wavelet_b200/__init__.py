"""wavelet_b200: a Blackwell-native post-training framework (SFT and online RL).

Packages: ``models`` (decoder architectures on flat parameters), ``ops``
(sm_100a kernels and their PyTorch references), ``parallel`` (process
groups, sharded optimizer state, fused collectives), ``trainer`` (SFT / RL
trainers, losses, checkpoints), ``data``, ``transport`` (filesystem rollout
and policy queues), ``orchestrator`` (rollout scheduling, rewards,
algorithms), ``inference`` (native batched generator and server), plus the
monitor, dashboard, debug and tools modules.
"""

__version__ = "0.1.0"
