"""TEST INFRASTRUCTURE ONLY -- the CPU oracle of mlx_nufft_b200.

This package restates the reference's (martinlachaine/mlx-nufft v0.1.3) CPU
algorithms for the NUFFT execute path in plain numpy / C so that the CUDA
library can be checked against them.  Only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline / `--impl reference` leg may import it, and only
as the checker or the timed CPU baseline; the product (mlx_nufft_b200) never
imports, links or calls anything here.

Parity pin: tests/test_oracle_pins.py checks every function below against
golden vectors produced by running the reference's own CPU code
(mlx_nufft/sizing.py, mlx_nufft/ref_t3.py, harness/gen.py) in the build
container -- see tests/golden/make_golden.py.

Modules
  port.py     numpy restatement: sizing, crit64 cells, types 1/2/3 pipelines
              (fp64), exact direct sums, rel_l2
  direct.c    OpenMP fp64 direct sum (same sum as port.direct_sum, faster)
  build.py    compiles direct.c into oracle/_build/liboracle.so
"""
