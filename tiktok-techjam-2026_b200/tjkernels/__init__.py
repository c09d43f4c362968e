"""B200 (sm_100a) engine for the causal pre-LN encoder forward.

A benchmark module opts in by routing its ``forward`` to ``forward(self, x,
valid_token_mask)``; everything else -- packing the module's weights into
fp16 tensor-core layouts, choosing a per-shape ``Plan``, running the CUDA
kernels of ``libtjb200.so`` and replaying the whole forward as a CUDA graph
-- happens behind that one call.  The module keeps owning its parameters
(the engine only reads them), so copying weights into it with
``load_state_dict`` needs nothing special.  ``get_engine`` returns the
engine cached on a module, ``reset_engines`` drops it, and ``select_plan``
shows which plan a shape gets.
"""

from .engine import forward, get_engine, reset_engines
from .plans import Plan, select_plan

__all__ = ["forward", "get_engine", "reset_engines", "Plan", "select_plan"]
