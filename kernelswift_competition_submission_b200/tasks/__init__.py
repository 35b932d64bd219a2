"""Drop-in task modules for the reference's evaluation harness.

Each file defines ``ModelNew``, ``get_inputs`` and ``get_init_inputs`` with the
signatures of the reference's ``<op>/v1/<op>.py`` and can be passed to its
``bench/auto_bench.py --v1_file``. The harness executes only imports, class and
function definitions and literal assignments at module level
(``bench/auto_bench.py:74-98``), so the package import happens inside
``_bootstrap()``.
"""
