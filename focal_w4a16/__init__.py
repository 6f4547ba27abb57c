"""Import-compatible alias: ``import focal_w4a16`` resolves to focal_b200.

Code written against the reference package (its tests and benches call
``focal_w4a16.w4a16_linear`` and friends) runs unchanged on the B200 kernels.
"""
from focal_b200 import *  # noqa: F401,F403
from focal_b200 import __all__  # noqa: F401
from focal_b200 import GROUP_SIZE, _ext  # noqa: F401
