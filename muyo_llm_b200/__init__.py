"""muyo_llm_b200: a B200-native (sm_100a) decode-step kernel set for muyo-llm's Qwen2 decode path.

The product is the C-ABI shared library ``_lib/libmuyo_cuda.so`` (include/muyo_cuda.h), built
in-tree by ``muyo_llm_b200.build``. This package holds its Python binding (``_abi``), the model
engine wrapper (``engine``), the multi-GPU row-sharded LM head (``shard``), seeded synthetic inputs
(``synth``) and a GGUF writer/reader (``gguf``).
"""
from ._abi import MuyoError, lib  # noqa: F401
from .build import build  # noqa: F401
