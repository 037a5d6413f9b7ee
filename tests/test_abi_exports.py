"""The C-ABI library loads without a GPU and exports every symbol include/deepinfer_cuda.h declares."""
import ctypes
import os
import subprocess

import pytest

import deepinfer_cuda as di


def test_header_declares_the_operator_table():
    syms = di.header_symbols()
    # QuantNative mirror (QuantizedMetal.cs:242-274) minus the gated-delta entries (not MoE)
    for name in ("di_quant_create", "di_quant_create_configured", "di_quant_destroy", "di_quant_residency_bytes",
                 "di_quant_residency_prepare", "di_quant_matrix_create", "di_quant_matrix_buffer",
                 "di_quant_matrix_destroy", "di_quant_batch", "di_quant_matvec", "di_quant_experts",
                 "di_quant_embedding", "di_moe_block", "di_moe_stack", "di_abi_version"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    if not os.path.exists(di.LIB_PATH):
        di.build()
    lib = ctypes.CDLL(di.LIB_PATH)
    missing = [s for s in di.header_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    assert set(di.SIGNATURES) == set(di.header_symbols())
    assert lib.di_abi_version() == 1


def test_library_targets_sm100a_only():
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", di.LIB_PATH], capture_output=True,
                         text=True).stdout
    assert "sm_100a" in out and "sm_90" not in out


def test_context_creation_fails_loudly_without_a_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    err = ctypes.create_string_buffer(2048)
    assert not di.lib().di_quant_create_configured(0, 1000, err, 2048)
    assert err.value  # an error message, never a silent CPU path


def test_invalid_configuration_rejected_before_device_use():
    err = ctypes.create_string_buffer(2048)
    assert not di.lib().di_quant_create_configured(2, 1000, err, 2048)
    assert b"Invalid residency configuration" in err.value
    assert not di.lib().di_quant_create_configured(1, 60001, err, 2048)
