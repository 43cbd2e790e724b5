"""B200 (sm_100a) attention kernels with the Python entry points of
KiritoHugh/attention_kernel_triton.

Each reference module has a same-named submodule here with the same launcher
signature; the work runs in hand-written CUDA behind the C ABI of
``include/akt.h`` (``libakt.so``).
"""
import importlib
import sys

# reference module name -> submodule of this package
DROPIN_MODULES = (
    "prefill_flash_attention",
    "prefill_flash_attention_var_len_padding",
    "decode_flash_attention_redundant",
    "decode_flash_attention_redundant_var_len_paged",
    "sparsetoken_decode_flash_attention_redundant",
    "sparsetoken_decode_flash_attention_redundant_var_len_paged",
    "magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm",
)


def install_dropin():
    """Make ``import <reference module name>`` resolve to this package's module.

    After this call, code written against the reference's top-level scripts
    (``from decode_flash_attention_redundant_var_len_paged import
    flash_attention_decode_paged``) runs the sm_100a kernels unchanged."""
    for name in DROPIN_MODULES:
        sys.modules[name] = importlib.import_module(f"{__name__}.{name}")
    return list(DROPIN_MODULES)
