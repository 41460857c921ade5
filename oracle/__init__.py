"""CPU oracle for the embedding-generation encoder path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library under
``jammi-ai_b200/`` and its Python loader) imports or executes this package;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may use it, and only as the checker / the timed CPU baseline.

The reference (Rust, candle 0.11) cannot be compiled in this environment, so
the oracle is a restatement of its arithmetic from the reference sources:

* ``oracle.bert``    -- ``crates/jammi-encoders/src/bert.rs``,
  ``layer_norm.rs``, ``mask.rs``, ``pooling.rs`` and the ``Linear`` call site
  ``crates/jammi-lora/src/wrapper.rs:29-42``.
* ``oracle.clip``    -- ``crates/jammi-ai/src/model/backend/open_clip_vit.rs``
  and ``l2_normalize`` in ``crates/jammi-ai/src/model/backend/candle.rs:425-438``.
* ``oracle.quant``   -- the int8 weight/activation format.  The reference has
  no int8 matmul; this format is defined by this project and its oracle is
  integer-exact (int64 accumulation).
* ``oracle.cpu_ref.cpp`` -- a C++/OpenMP f32 restatement used as the timed
  CPU baseline (built into ``oracle/_build``).

Pinning: the float restatement is checked against (1) the reference's own
known-answer tests for pooling (``crates/jammi-encoders/tests/it/pooling.rs``)
and padding (``tests/it/bert.rs:260-315``), and (2) golden vectors produced by
HuggingFace ``transformers`` (the implementation the reference's own parity
test mirrors via candle-transformers) on seeded tiny fixtures, committed under
``tests/golden/`` with the script that made them.  The int8 path has no
reference counterpart and is "parity unpinned" against the reference: it is
pinned against integer-exact arithmetic instead.
"""
