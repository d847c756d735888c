"""B200 decode backend for the xiaoju-pipe Qwen3.5-style hybrid decoder.

The product is the C-ABI library ``csrc/libxj_cuda.so`` (declared in ``include/xj_cuda.h``); this
package only holds its Python front end (``xjcuda``) and the synthetic-model writer used by tests and
the benchmark (``synth``). Load it by path, since the folder name is not a Python identifier::

    spec = importlib.util.spec_from_file_location(
        "xjb200", "meta-work_b200/__init__.py", submodule_search_locations=["meta-work_b200"])
"""
