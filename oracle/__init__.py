"""CPU oracle for the Qwen3 per-step hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or the timed CPU baseline.

The oracle is a plain-PyTorch (CPU) restatement of the reference engine's
forward pass (yijichar/AWesome_ACceleration ``model/model.py`` and
``llm.py``), with the three flash-attn entry points restated from their
documented semantics.  It is pinned against golden vectors produced by running
the reference's own ``LLM._prefill`` / ``LLM._decode_step`` code (see
``tests/golden/make_golden.py``).  The flash-attn arithmetic itself cannot run
on a CPU; its restatement is pinned separately against the installed
flash-attn library on a GPU where that library runs.
"""
