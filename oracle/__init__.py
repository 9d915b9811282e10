"""CPU oracle for the MTP speculative-decode MoE path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithms that the CUDA
kernels in home_seek_b200 replace. Each function cites the reference
file:line it follows (paths inside the home-seek project). It is used only as
the checker: by tests/, by __graft_entry__.smoke(), and by bench.py's CPU
baseline leg. The product path (home_seek_b200) never imports it and fails
loudly when its CUDA library is missing.

Pinning: the restatement is checked against golden vectors produced by running
the reference's own code (home_seek.router, home_seek.fused_moe,
HomeSeekInferenceEngine._compute_hash_experts / _mtp_verify_batched,
tests/_reference.py) on the same seeded inputs; see tests/golden/make_golden.py
and tests/test_oracle_golden.py. Rejection sampling has no counterpart in the
reference; its oracle (oracle.accept.rejection) is a restatement of standard
speculative sampling and is parity-unpinned by the reference.
"""
