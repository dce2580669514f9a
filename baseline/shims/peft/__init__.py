"""Import-only stand-in for the ``peft`` package, used by the reference arm of
``bench.py`` only.

The reference framework imports ``peft`` at module level
(``wavelet/trainer/model.py:17-24``, ``wavelet/transport/policy.py:17``), but
``peft`` is neither in this image nor in its offline wheelhouse.  The dense SFT
configuration that the reference arm runs sets ``lora: null``, so no function
below is ever called on that path; each one raises if it is.  ``PeftModel`` is
only used there in ``isinstance`` checks, which a plain class answers with
``False`` for every real model.
"""

from __future__ import annotations

import enum

__version__ = "0.0.0+wavelet-b200-import-shim"


class _Unavailable(RuntimeError):
    pass


def _refuse(name: str):
    def f(*args, **kwargs):
        raise _Unavailable(f"peft.{name} called, but only an import shim of peft is installed")

    f.__name__ = name
    return f


class PeftModel:  # never instantiated on the dense path
    @classmethod
    def from_pretrained(cls, *args, **kwargs):
        raise _Unavailable("peft.PeftModel.from_pretrained called, but only an import shim of peft is installed")


class PeftConfig:
    pass


class LoraConfig(PeftConfig):
    def __init__(self, *args, **kwargs):
        raise _Unavailable("peft.LoraConfig called, but only an import shim of peft is installed")


class TaskType(str, enum.Enum):
    CAUSAL_LM = "CAUSAL_LM"


get_peft_model = _refuse("get_peft_model")
get_peft_model_state_dict = _refuse("get_peft_model_state_dict")
set_peft_model_state_dict = _refuse("set_peft_model_state_dict")
prepare_model_for_kbit_training = _refuse("prepare_model_for_kbit_training")
