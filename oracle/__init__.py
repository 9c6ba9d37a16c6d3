"""CPU oracle for the B200 decode path -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it.  The library (``llm_compiler_3_b200``) must never
import it, and fails loudly when its CUDA extension is missing instead of
falling back to anything here.

It restates, in plain PyTorch on the CPU with FP32 arithmetic over FP16-stored
tensors, the computation LLM_Compiler_3 captures and checks against
(``examples/llama/verify.py:80-82``, ``docs/DESIGN.md:404-405``): the Hugging
Face decoder layer the reference captures, evaluated as a decode step with a
flat KV cache.  ``oracle/decode.py`` cites the reference file:line each function
follows; ``tests/golden/`` pins it against ``transformers`` itself and against
the reference's own known-answer tests.
"""
from .decode import *  # noqa: F401,F403
from .graph import run_graph_plan  # noqa: F401
