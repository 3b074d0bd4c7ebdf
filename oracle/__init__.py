"""CPU oracle for the sparse 3-D refinement step -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the reference algorithm of every stage of PromptMoGe's refinement step
(voxelisation, voxel dedup / pooling cache, neighbour maps, the int8 refiner forward, the trimmed least-squares
metric fit).  It is the checker the CUDA path is compared against, and the CPU baseline that ``bench.py`` times.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may import it; the
product path (``promptmoge_b200``) never does.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own pure-PyTorch path (its bundled FlexGEMM
fallback plus ``moge.model.v3`` / ``prompt_stem.fit_scale_shift``) on seeded synthetic inputs and commits the outputs
under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle against them.
"""
