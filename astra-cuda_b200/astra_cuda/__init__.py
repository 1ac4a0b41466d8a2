"""astra_cuda -- B200-native (sm_100a) lock-step double-auction matching engine.

Drop-in for the ``order_matching`` submodule of nlyu1/astra-cuda's
``astra_cuda`` extension (src/pybind/bindings.cc:16-21).  The game API of that
extension (``load_game``, ``State``, ...) is not part of this package.
"""
__version__ = "0.0.2"  # bindings.cc:10

from . import order_matching  # noqa: E402,F401
