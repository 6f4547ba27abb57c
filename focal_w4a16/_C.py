"""``focal_w4a16._C``: the extension module name the reference package imports
(focal_w4a16/__init__.py:25-27 imports it lazily and calls its w4a16_linear).

Here the name is served by focal_b200's PyTorch extension (focal_b200/_C, the
thin shim over libfocal_b200.so), so code that imports the reference's module
directly gets the B200 kernels with no edit.  Importing it fails loudly when the
extension has not been built; there is no fallback.
"""
from focal_b200 import _ext as _load_extension

_ext = _load_extension()


def __getattr__(name):
    return getattr(_ext, name)


w4a16_linear = _ext.w4a16_linear
