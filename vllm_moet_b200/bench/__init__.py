"""Benchmark harness: recipes (YAML) -> runs -> schema'd, hash-bound results.

    python -m vllm_moet_b200.bench run  <recipe.yaml | name> [--out results/]
    python -m vllm_moet_b200.bench lint <results.json ...>
    python -m vllm_moet_b200.bench render <results.json ...>

A recipe names a model preset, its overrides, the engine options and a list
of probes (``decode`` at given stream counts, ``prefill`` at given lengths,
``coherence``: greedy outputs identical across two runs).  A result file
(schema 2) records every measurement together with the sha256 of the recipe,
the git commit, the native source fingerprint and the GPU name, so a number
can always be traced to exactly what produced it; ``lint`` refuses results
whose recipe hash does not match the recipe file or whose fields are missing
(the reference's bench runner / lint / render, bench/runner/*.py).
"""
