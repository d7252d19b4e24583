"""B200-native paged-decode attention for the llm-serving engine.

Put this directory on ``sys.path``: the modules then resolve under the reference's own names
(``model.triton_decode``, ``model.paged``, ``serve.block_manager``). The sm_100a kernels and
their C ABI live in ``csrc/`` and build into ``libpaged_decode.so`` (``build.py``).
"""
