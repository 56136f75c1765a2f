"""Host-side contract of ``sparse_attention`` (hilberta/sparse_kernel.py:188-339)
on tensor-property fakes, without touching CUDA: the reference's cases of
tests/test_sparse_kernel_contract.py (same error types and message substrings)
plus the pairing requirement of this package's execution."""

from __future__ import annotations

import unittest

import torch

from hilberta_b200.sparse_kernel import _check_inputs, sparse_attention
from tests.test_paired_kernel_contract import TensorProperties


class SparseContract(unittest.TestCase):
    def setUp(self):
        shape = (1, 2, 512, 128)
        native = (131072, 128, 256, 1)
        self.q = TensorProperties(shape, native, pointer=1_000_000)
        self.k = TensorProperties(shape, pointer=2_000_000)
        self.v = TensorProperties(shape, native, pointer=3_000_000)
        self.ids = TensorProperties((6, 5), dtype=torch.int32, pointer=4_000_000)
        self.counts = TensorProperties((6,), dtype=torch.int32, pointer=5_000_000)
        self.out = TensorProperties(shape, native, pointer=6_000_000)

    def check(self, **changes):
        values = dict(q=self.q, k=self.k, v=self.v, kv_indices=self.ids, kv_counts=self.counts, global_tokens=128,
                      block_size=64, out=self.out)
        values.update(changes)
        return _check_inputs(**values)

    def test_native_output_and_mixed_input_strides(self):
        self.check()

    def test_head_major_output(self):
        self.check(out=TensorProperties(self.q.shape, pointer=6_000_000))

    def test_aliases_are_rejected(self):
        for ptr in (self.q.pointer, self.k.pointer + 1024, self.ids.pointer):
            with self.subTest(ptr=ptr):
                self.out.pointer = ptr
                with self.assertRaisesRegex(ValueError, "alias"):
                    self.check()

    def test_overlapping_and_zero_stride_outputs_are_rejected(self):
        self.out.strides = (131072, 128, 128, 1)
        with self.assertRaisesRegex(ValueError, "non-overlapping"):
            self.check()
        self.out.strides = (0, 128, 256, 1)
        with self.assertRaisesRegex(ValueError, "positive"):
            self.check()

    def test_gradients(self):
        self.q.requires_grad = True
        with torch.enable_grad(), self.assertRaisesRegex(ValueError, "inference-only"):
            self.check()
        with torch.no_grad():
            self.check()
        self.q.requires_grad = False
        self.out.requires_grad = True
        with torch.enable_grad(), self.assertRaisesRegex(ValueError, "gradients"):
            self.check()

    def test_integer_fields_and_shapes(self):
        for value in (128.0, True):
            with self.subTest(value=value), self.assertRaises(TypeError):
                self.check(global_tokens=value)
        with self.assertRaisesRegex(ValueError, "align"):
            self.check(global_tokens=100)
        with self.assertRaisesRegex(ValueError, "partition"):
            self.check(kv_indices=TensorProperties((5, 5), dtype=torch.int32, pointer=4_000_000))
        with self.assertRaisesRegex(ValueError, "int32"):
            self.check(kv_counts=TensorProperties((6,), dtype=torch.int64, pointer=5_000_000))
        self.q.shape = self.k.shape = self.v.shape = (0, 2, 512, 128)
        with self.assertRaisesRegex(ValueError, "nonempty"):
            self.check(out=None)

    def test_tuning_and_scale_rejected_without_device_work(self):
        args = (self.q, self.k, self.v, self.ids, self.counts)
        with self.assertRaisesRegex(TypeError, "never a tensor"):
            sparse_attention(*args, global_tokens=128, scale=torch.tensor(1.0))
        with self.assertRaisesRegex(ValueError, "global_strategy"):
            sparse_attention(*args, global_tokens=128, global_strategy="dense")
        with self.assertRaisesRegex(ValueError, "Supported tuning"):
            sparse_attention(*args, global_tokens=128, query_block_size=128)
        with self.assertRaisesRegex(ValueError, "positive and finite"):
            sparse_attention(*args, global_tokens=128, scale=-1.0)

    def test_pairing_needs_128_alignment(self):
        shape = (1, 2, 576, 128)
        q = TensorProperties(shape, pointer=1_000_000)
        k = TensorProperties(shape, pointer=2_000_000)
        v = TensorProperties(shape, pointer=3_000_000)
        ids = TensorProperties((7, 5), dtype=torch.int32, pointer=4_000_000)
        counts = TensorProperties((7,), dtype=torch.int32, pointer=5_000_000)
        with self.assertRaisesRegex(NotImplementedError, "multiples of 128"):
            sparse_attention(q, k, v, ids, counts, global_tokens=128)
