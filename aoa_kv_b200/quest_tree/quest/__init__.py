"""Drop-in ``quest`` package backed by libaoakv.so.

Put ``aoa_kv_b200/quest_tree`` first on sys.path (or register it as a kernel
tree in latency/bench_latency.py) and ``import quest.utils`` resolves to the
B200 library with the reference's names and signatures
(kernels/aoa_kv/quest/utils/__init__.py:11-23, ops/csrc/bsk_ops.cu:4-19).

The scoring mode of the tree is chosen with AOAKV_SCORE_MODE ("aoakv", the
default, like kernels/aoa_kv; "quest" like kernels/quest_orig).
"""
import sys
from pathlib import Path

try:
    import aoa_kv_b200  # noqa: F401
except ImportError:  # the tree sits inside the repository: make its root importable
    sys.path.insert(0, str(Path(__file__).resolve().parents[3]))

from . import _kernels, utils  # noqa: E402,F401

__version__ = "0.0.1"
__all__ = ["LlamaForCausalLM"]


def __getattr__(name):
    if name == "LlamaForCausalLM":
        raise NotImplementedError(
            "quest.LlamaForCausalLM (quest/models/llama.py) is not provided by this tree; "
            "the sparse-decode operators are (quest.utils)")
    raise AttributeError(name)
