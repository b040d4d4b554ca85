"""eagle_b200: a B200-native (sm_100a) backend for eagle's until-done hot path.

The engine lives in ``libeagle_b200.so`` (hand-written CUDA behind eagle's
``eagle-backend/1`` C seam, declared in ``include/eagle_b200.h``); this package is
its eagle-shaped Python face. Importing it loads nothing; the first call loads the
library and fails loudly (``BackendUnavailable``) when it is not built.
"""

from ._abi import BackendError, BackendUnavailable, BackendUnsupported
from ._api import (Compactor, CompactSum, Model, Reducer, Runner, RunReport, SimResult, StagedRunner, cell_op,
                   compact, entry, gambler, lorenz, mask_count, oscillator, reduce, reorder, reorder_classes, restore, simulate,
                   until_done)

__all__ = ["BackendError", "BackendUnavailable", "BackendUnsupported", "Compactor", "CompactSum", "Model", "Reducer",
           "Runner", "RunReport", "SimResult", "StagedRunner", "cell_op", "compact", "entry", "gambler", "lorenz",
           "mask_count", "oscillator", "reduce", "reorder", "reorder_classes", "restore", "simulate", "until_done"]
