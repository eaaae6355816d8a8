"""Import the in-tree native extension (mirrors ``complex_conv2d/_extension.py:1-12``).

There is no CPU or eager fallback: if the extension is not built, importing
the package fails loudly.
"""

try:
    from . import _C as cutlass_complex_conv
except ImportError as exc:
    raise ImportError(
        "The cutlass-complex-conv B200 extension is not built. "
        "Build it from the repository root with "
        "`python cutlass-complex-conv_b200/build.py` "
        "(or `python -c 'import __graft_entry__ as g; g.build()'`)."
    ) from exc

__all__ = ["cutlass_complex_conv"]
