"""Test infrastructure: CPU restatement of the reference decode path and the
reference's own PyTorch path (HF Qwen3ForCausalLM).  Used only by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg -- never by the
qwen_megakernel_b200 product code."""
