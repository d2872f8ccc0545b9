"""Import name of the reference project, served by ``lsso_b200``.

``import lsso`` / ``from lsso.ball import cuda`` resolve to the very same
module objects as ``lsso_b200`` (so monkeypatching either is the same).
"""

import sys as _sys

import lsso_b200 as _impl
import lsso_b200.ball as _ball
import lsso_b200.ball.config as _config
import lsso_b200.ball.cuda as _cuda
import lsso_b200.ball.model as _model
import lsso_b200.ball.reference as _reference

_sys.modules[__name__ + ".ball"] = _ball
_sys.modules[__name__ + ".ball.config"] = _config
_sys.modules[__name__ + ".ball.cuda"] = _cuda
_sys.modules[__name__ + ".ball.model"] = _model
_sys.modules[__name__ + ".ball.reference"] = _reference
ball = _ball

from lsso_b200 import CoreMode, LSSO, LSSOConfig, __version__  # noqa: E402

__all__ = ["CoreMode", "LSSO", "LSSOConfig", "__version__"]
