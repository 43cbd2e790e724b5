"""Drop-in surface: module names, function names and signatures match the reference launchers."""
import inspect
import sys

import attention_kernel_triton_b200 as akt

# reference signatures (DR:233, DP:228, SD:127, SP:170, MP:166)
EXPECTED = {
    "prefill_flash_attention": ("flash_attention_prefill",
                                ["Q", "K", "V", "causal", "softmax_scale", "GQA_group_size"]),
    "prefill_flash_attention_var_len_padding": (
        "flash_attention_prefill", ["Q", "K", "V", "causal", "softmax_scale", "GQA_group_size", "varlen"]),
    "decode_flash_attention_redundant": ("flash_attention_decode", ["q", "K", "V", "softmax_scale", "GQA_group_size"]),
    "decode_flash_attention_redundant_var_len_paged": (
        "flash_attention_decode_paged", ["q", "paged_kv_cache", "kv_page_indptr", "kv_page_indices", "kv_last_page_len"]),
    "sparsetoken_decode_flash_attention_redundant": (
        "sparsetoken_flash_attention_decode",
        ["q", "K", "V", "sparse_ind", "sparse_nnz", "softmax_scale", "GQA_group_size"]),
    "sparsetoken_decode_flash_attention_redundant_var_len_paged": (
        "sparsetoken_flash_attention_decode_paged",
        ["q", "paged_kv_cache", "kv_page_indptr", "kv_page_indices", "sparse_ind", "sparse_nnz"]),
    "magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm": (
        "magicpig_sparsetoken_flash_attention_decode_paged",
        ["q", "paged_kv_cache", "kv_page_indptr", "kv_page_indices", "sparse_ind", "sparse_nnz", "K", "L"]),
}


def test_install_dropin_resolves_reference_module_names():
    names = akt.install_dropin()
    try:
        assert set(EXPECTED) <= set(names)
        for mod, (fn, params) in EXPECTED.items():
            m = __import__(mod)
            assert m.__name__.startswith("attention_kernel_triton_b200.")
            f = getattr(m, fn)
            assert list(inspect.signature(f).parameters) == params
    finally:
        for mod in EXPECTED:
            sys.modules.pop(mod, None)


def test_default_arguments_match_reference():
    from attention_kernel_triton_b200.decode_flash_attention_redundant import flash_attention_decode
    assert inspect.signature(flash_attention_decode).parameters["GQA_group_size"].default == 1
