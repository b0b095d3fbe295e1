"""B200-native (sm_100a) transformer-layer library.

The compute lives in ``libb200_llm.so`` (CUDA kernels + C++ engine behind the
C ABI of ``include/b200_llm.h``); :mod:`atb_llm_study_b200.capi` binds it.
Build it with ``python -m atb_llm_study_b200.build``.
"""

from .capi import B200Error, check, lib  # noqa: F401
