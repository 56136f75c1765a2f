"""Host-side contract of ``paired_attention`` without touching CUDA: tensor
property fakes, the native launch patched out.  Mirrors the reference's
``tests/test_paired_kernel_contract.py`` and ``tests/test_sparse_kernel_contract.py``
cases (same error types and message substrings)."""

from __future__ import annotations

import unittest
from types import SimpleNamespace
from unittest.mock import MagicMock, patch

import torch

from hilberta_b200.paired_kernel import paired_attention
from hilberta_b200.sparse_kernel import _non_overlapping_strides, _tensor_byte_span


class TensorProperties:
    """Shape/stride/pointer-only stand-in for a CUDA tensor."""

    def __init__(self, shape, strides=None, dtype=torch.bfloat16, pointer=1_000_000, device="cuda:0", requires_grad=False):
        self.shape = tuple(shape)
        self.ndim = len(shape)
        self.dtype = dtype
        self.device = torch.device(device)
        self.is_cuda = self.device.type == "cuda"
        self.requires_grad = requires_grad
        self.pointer = pointer
        if strides is None:
            strides, running = [], 1
            for size in reversed(shape):
                strides.insert(0, running)
                running *= size
        self.strides = tuple(strides)

    def stride(self, dim=None):
        return self.strides if dim is None else self.strides[dim]

    def data_ptr(self):
        return self.pointer

    def element_size(self):
        return 4 if self.dtype == torch.int32 else 2

    def is_contiguous(self):
        running = 1
        for size, stride in zip(reversed(self.shape), reversed(self.strides)):
            if size > 1 and stride != running:
                return False
            running *= size
        return True


class PairedContract(unittest.TestCase):
    def setUp(self):
        shape = (1, 2, 512, 128)
        native = (131072, 128, 256, 1)
        self.q = TensorProperties(shape, native, pointer=1_000_000)
        self.k = TensorProperties(shape, pointer=2_000_000)
        self.v = TensorProperties(shape, native, pointer=3_000_000)
        self.meta = SimpleNamespace(
            tokens=512,
            global_tokens=128,
            key_block_size=64,
            kv_indices=TensorProperties((3, 5), dtype=torch.int32, pointer=4_000_000),
            kv_flags=TensorProperties((3, 5), dtype=torch.int32, pointer=5_000_000),
            kv_counts=TensorProperties((3,), dtype=torch.int32, pointer=6_000_000),
        )
        self.out = TensorProperties(shape, native, pointer=7_000_000)

    def call(self, **kwargs):
        launch = MagicMock()
        with patch("hilberta_b200.paired_kernel._launch", launch):
            res = paired_attention(self.q, self.k, self.v, self.meta, out=self.out, global_strategy="triton", **kwargs)
        self.last_launch = launch
        return res

    def test_mixed_stride_native_output(self):
        self.assertIs(self.call(), self.out)
        args = self.last_launch.call_args[0]
        self.assertEqual(args[5:8], (512, 128, 128**-0.5))

    def test_flash_strategy_uses_the_same_single_launch(self):
        launch = MagicMock()
        with patch("hilberta_b200.paired_kernel._launch", launch):
            paired_attention(self.q, self.k, self.v, self.meta, out=self.out, global_strategy="flash")
        self.assertEqual(launch.call_count, 1)

    def test_input_and_metadata_output_alias_rejected(self):
        for source in (self.q, self.k, self.v, self.meta.kv_indices, self.meta.kv_flags, self.meta.kv_counts):
            with self.subTest(source=source.pointer), self.assertRaisesRegex(ValueError, "alias"):
                self.out.pointer = source.pointer
                self.call()

    def test_partial_alias(self):
        self.out.pointer = self.k.pointer + 64
        with self.assertRaisesRegex(ValueError, "alias"):
            self.call()

    def test_overlap_and_zero_stride_output(self):
        for strides in ((131072, 128, 128, 1), (0, 128, 256, 1)):
            self.out.strides = strides
            with self.assertRaisesRegex(ValueError, "non-overlapping"):
                self.call()

    def test_grad_inputs_outputs(self):
        self.q.requires_grad = True
        with torch.enable_grad(), self.assertRaisesRegex(ValueError, "Inference"):
            self.call()
        with torch.no_grad():
            self.call()
        self.q.requires_grad = False
        self.out.requires_grad = True
        with torch.enable_grad(), self.assertRaisesRegex(ValueError, "gradients"):
            self.call()

    def test_tensor_scale_not_transferred(self):
        with self.assertRaisesRegex(TypeError, "never a tensor"):
            self.call(scale=torch.tensor(1.0))

    def test_scale_must_be_positive_finite(self):
        for s in (0.0, -1.0, float("inf"), float("nan")):
            with self.subTest(scale=s), self.assertRaisesRegex(ValueError, "Positive finite scale"):
                self.call(scale=s)

    def test_tuning_rejects_noninteger(self):
        for value in (4.0, True):
            with self.assertRaisesRegex(TypeError, "Integer"):
                self.call(num_warps=value)

    def test_tuning_range(self):
        with self.assertRaisesRegex(ValueError, "Invalid launch tuning"):
            self.call(num_warps=2)
        with self.assertRaisesRegex(ValueError, "Invalid launch tuning"):
            self.call(num_stages=5)

    def test_bad_strategy(self):
        with self.assertRaisesRegex(ValueError, "Invalid global strategy"):
            launch = MagicMock()
            with patch("hilberta_b200.paired_kernel._launch", launch):
                paired_attention(self.q, self.k, self.v, self.meta, out=self.out, global_strategy="sdpa")

    def test_wrong_device(self):
        self.meta.kv_flags.device = torch.device("cuda:1")
        with self.assertRaisesRegex(ValueError, "CUDA"):
            self.call()

    def test_cpu_inputs_rejected(self):
        self.q.device = torch.device("cpu")
        self.q.is_cuda = False
        with self.assertRaisesRegex(ValueError, "CUDA"):
            self.call()

    def test_metadata_shapes(self):
        self.meta.kv_flags.shape = (3, 4)
        with self.assertRaisesRegex(ValueError, "shape"):
            self.call()

    def test_metadata_dtype(self):
        self.meta.kv_counts.dtype = torch.int64
        with self.assertRaisesRegex(ValueError, "int32"):
            self.call()

    def test_metadata_alignment(self):
        self.meta.global_tokens = 64
        with self.assertRaisesRegex(ValueError, "alignment"):
            self.call()

    def test_metadata_integer_fields(self):
        self.meta.tokens = 512.0
        with self.assertRaisesRegex(TypeError, "Integer metadata"):
            self.call()

    def test_negative_input_stride(self):
        self.k.strides = (131072, -128, 256, 1)
        with self.assertRaisesRegex(ValueError, "Positive"):
            self.call()

    def test_head_dim_and_dtype(self):
        for shape in ((1, 2, 512, 96),):
            self.q.shape = self.k.shape = self.v.shape = shape
            with self.assertRaisesRegex(ValueError, "D64 or128"):
                self.call()
        self.q.shape = self.k.shape = self.v.shape = (1, 2, 512, 128)
        self.v.dtype = torch.float16
        with self.assertRaisesRegex(TypeError, "BF16/FP16"):
            self.call()

    def test_empty_rejected(self):
        self.q.shape = self.k.shape = self.v.shape = (0, 2, 512, 128)
        with self.assertRaisesRegex(ValueError, "nonempty"):
            self.call()


class SpanHelpers(unittest.TestCase):
    def test_byte_span_and_overlap(self):
        t = TensorProperties((1, 2, 512, 128), (131072, 128, 256, 1), pointer=1000)
        self.assertEqual(_tensor_byte_span(t), (1000, 1000 + 2 * (1 + 511 * 256 + 128 + 127)))
        self.assertTrue(_non_overlapping_strides(t))
        t.strides = (131072, 128, 128, 1)
        self.assertFalse(_non_overlapping_strides(t))


if __name__ == "__main__":
    unittest.main()
