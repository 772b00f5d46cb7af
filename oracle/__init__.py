"""CPU oracle for the HSD verification hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU, the algorithm
of the reference's verification path (whlscut/HSD,
``hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py`` and
``hsd/hunyuan_ocr_pipeline/modeling_hunyuan_vl_hsd.py``) so that the CUDA
kernels of :mod:`hsd_b200` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and its
``--impl reference`` arm) may import it, and only as the checker or the
timed CPU baseline -- never as the thing measured or shipped.  The product
path (:mod:`hsd_b200`) never imports this package and has no CPU fallback.

Modules
-------
``kmp``        failure table, KMP search and continuation trie (D:543-618)
``blockmask``  dense mask -> 128x64 tile classification (D:94-106, D:148-153)
``masks``      packed-mask assembly from segment descriptors (RD:234-245,
               D:1634-1667, D:1737-1748)
``attention``  fp32 masked GQA attention with LSE (D:72-146)
``accept``     per-block acceptance, tree walk, stop rules, re-alignment
               (D:1103-1336, D:1426-1567)
``compact``    live/keep columns, compaction rule, index_select (D:1669-1735,
               H:2237-2285)

Parity pinning: ``tests/golden/make_golden.py`` imports the reference module
in a container where it is present and records its outputs (KMP tables,
matches and tries; FlexAttention block masks; FlexAttention outputs on seeded
inputs).  ``tests/test_oracle_golden.py`` checks this package against those
fixtures.  The acceptance loop and compaction are inline code inside the
reference's ``batch_generate`` and cannot be imported; they are restated
line by line here with citations, and pinned through the imported KMP
functions they call.

Citations use ``D`` = hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py,
``H`` = hsd/hunyuan_ocr_pipeline/modeling_hunyuan_vl_hsd.py,
``RD`` = hsd/dots_ocr_pipeline/run_dots_ocr_hsd.py.
"""
