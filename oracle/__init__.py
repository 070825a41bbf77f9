"""CPU oracle for the SKCQ codebook-build and codebook-expert-forward paths.

TEST INFRASTRUCTURE ONLY. This package is a numpy restatement of the
reference algorithm (levzlotnik/SKCQ, ``skcq/codebook/*.py`` and
``skcq/codebook_experts.py``). It exists to check the CUDA path: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline -- never as the thing measured or shipped.
The product package ``skcq_b200`` never imports it.

Every function cites the reference ``file:line`` it restates. All arithmetic
is float32 (the reference runs ``w.float()``), so results agree with the
reference up to the rounding order of BLAS / torch reductions; the parity
pins in ``tests/test_oracle_golden.py`` check that against vectors produced by
the reference itself (``tests/golden/make_golden.py``).

Two inputs are taken from torch rather than restated, because they come from
torch's own random generators, not from SKCQ: the scrambled-Sobol initial
directions (``skcq/codebook/kmeans.py:69-74``, ``torch.quasirandom.SobolEngine``,
seed 42) and the Forgy permutation (``kmeans.py:201``, ``torch.randperm`` on
the global generator). The oracle's fit functions take them as arguments.
"""

from oracle.kmeans import (  # noqa: F401
    assign_cosine,
    assign_l2,
    fit_cosine,
    fit_euclidean,
    normalize_rows,
    scores_cosine,
    scores_l2,
)
