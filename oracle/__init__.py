"""CPU oracle of karpo-decision's packed prefill forward: a numpy restatement of the reference algorithm, used only as
the checker (tests, ``__graft_entry__.smoke``) and as the timed CPU baseline of ``bench.py``. Test infrastructure,
never the product path: nothing under ``karpo_decision_b200`` imports it.

Pinned against the reference itself: ``tests/golden/make_golden.py`` runs the reference's own ``families.*.Packed`` and
``Readout`` (imported from the reference source tree, CPU, float32) over the same seeded weights and packs, and
``tests/test_oracle_golden.py`` checks this restatement against those fixtures.
"""

from .packed import (  # noqa: F401
    attention_varlen,
    bf16,
    e4m3_rows,
    gemma_forward,
    qwen_forward,
    readout,
    rms_norm,
    rope_tables,
)
