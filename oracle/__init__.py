"""CPU oracle for the Q8_0 Llama-2 decode path -- TEST INFRASTRUCTURE ONLY.

A restatement of ZeroR0R/tensor-inference-runtime's CPU path (Rust) used as
the checker for the CUDA implementation.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may
import this package; the product never calls it.

* ``oracle.liboracle.so`` (``oracle.c``): the arithmetic -- matvecs,
  quantisation, norms, rope, attention, the forward pass and greedy decode.
* ``oracle.gguf_ref``: the GGUF reader (``src/reader.rs``, ``src/lib.rs``
  ``load_model``) in plain Python.

Parity status: pinned against the reference's own known-answer unit tests;
whole-model outputs are not pinned by running the reference (no Rust
toolchain is available to build it).
"""
from .binding import Oracle, load_oracle, ORACLE_DIR  # noqa: F401
