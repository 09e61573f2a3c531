"""The oracle: a CPU restatement of the reference's algorithms for this path.

TEST INFRASTRUCTURE ONLY. Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg (``--impl reference`` and the ``cpu_baseline`` field) import this package, and
only to check results or as the timed CPU reference implementation; the product path
(kta_b200) never imports, calls or links anything here.

Contents, each citing the reference code it restates (paths within kernel-template-agent):

- ``numerics``: exact widening of bf16 / f16 / e4m3 bit patterns to float64 (numpy).
- ``gemm``: the GEMM case statements ``C = A @ B`` (knowledge/seed/cases/gemm_fp16.yaml:8)
  and ``C = A @ B.T`` evaluated in FP64 as src/kta/checks/scripts/ref_torch.py:28-38 does.
- ``fp8``: the block-scaled FP8 statement (dequantise, then FP64 product) and the e4m3
  quantiser of the input generator.
- ``attention``: causal attention forward with log-sum-exp, and GQA decode with the
  split-KV partial / log-sum-exp combine of perfmodel/testset/gen.py:417-590.
- ``statement``: the reference's statement runner (ref_torch.py:17-45) on the CPU.

Pinning: tests/golden holds fixtures generated in a container where the reference's Python
is importable (tests/golden/make_golden.py): the reference's own input generators, its own
ref_torch.py run on the CPU, and its compare_output / library_verdict / bound. The oracle is
checked against them in tests/test_oracle_golden.py. tests/golden/kernels.npz holds the
outputs of the reference's own TileLang kernels (fa_forward, decode_partial + decode_combine,
fp8gemm; perfmodel/testset/gen.py) run on a B200 by tests/golden/make_kernel_golden.py; the
non-causal attention, the split / combine decode and the unscaled FP8 product here match them
within the kernels' f16 roundings (same test file). The causal mask, the LSE output, the FP8
block scales and variable decode lengths have no reference kernel: the cases' statements
define them, and the statement runner fixtures pin the oracle to those.
"""
