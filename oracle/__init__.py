"""Oracle: a CPU restatement of LateFuse's late-fusion LoRA serving path.

TEST INFRASTRUCTURE ONLY.  Nothing in the ``latefuse_b200`` package imports
this package; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm may import it, and only as the checker or as the timed
CPU baseline -- never as the thing measured on the GPU or shipped.

Each function restates one piece of the reference algorithm in plain PyTorch on
the CPU and cites the reference file:line it follows (paths within the
ashutoshrdwivedi/LateFuse project).  The restatement is pinned against golden
vectors produced by running the reference itself (``tests/golden/make_golden.py``
imports the reference; the fixtures it writes are committed under
``tests/golden/``), and ``tests/test_oracle_golden.py`` checks the oracle against
every fixture.

The third-party arithmetic underneath the reference -- ``torch.bmm`` /
``index_select`` / ``normalize`` (torch 2.11) and the HuggingFace encoder
forward (transformers; the reference pins 4.57.6, this image has 5.5.0) -- is
used here the same way the reference uses it.
"""
