"""Paged-KV decode path on B200: the drop-in for the reference's ``model/triton_decode.py``
and ``model/paged.py`` (import the submodules: ``model.triton_decode``, ``model.paged``)."""
