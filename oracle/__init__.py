"""CPU oracle for the live-reshard path -- TEST INFRASTRUCTURE ONLY.

A restatement in plain Python/numpy of Suika's schedule_param_transfer and execute_param_transfer
(Suika/migration.py:322-556), used as the checker for the CUDA path. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import it; the product package
(suika_b200) never does, and has no CPU path of its own.

Parity is pinned: tests/test_oracle_golden.py checks this restatement against golden digests
produced by running the reference itself on CPU/gloo ranks (tests/golden/make_golden.py).

Modules:
  restate     schedule_param_transfer / execute_param_transfer on numpy (the checker);
  activation  the cross-stage activation exchange of Suika/pipeline_parallel.py:665-836, pinned by
              tests/golden/act_golden.json (tests/golden/make_act_golden.py);
  nccl_port   execute_param_transfer as the reference runs it on GPUs (torch.distributed P2P per
              tensor), the library baseline bench.py times; pinned on gloo ranks by
              tests/test_reference_port.py.
"""
