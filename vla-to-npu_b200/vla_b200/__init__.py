"""vla_b200 — B200 (sm_100a) implementation of the SmolVLA bf16 inference hot
path of xl434/vla-to-npu, behind the reference's block-builder and per-op
entry points."""
