"""svllm_ops.rms_norm keeps the reference's contract: the reference's own op test
(tests/python/test_rms_norm.py:9-66), same shapes, seeds, oracle, tolerance and error fragments,
run on CPU and (marked gpu) on the sm_100a kernel. On CUDA it must also be bit-identical to the
reference's own CUDA kernel, built from its sources for sm_100a (oracle/_ref): the op's bar
allows one bf16 ulp, and the kernels reproduce the reference's summation order and rsqrtf so
that they need none."""

import pytest
import svllm_ops
import torch
import torch.nn.functional as F
from conftest import assert_bf16_within_ulp, assert_close_bf16, random_bf16

import oracle

EPS = 1e-6

SHAPES = [
    (0, 1024),  # an empty batch: no kernel launch
    (1, 128),  # one token, Qwen3 head_dim for QK-norm
    (4, 64),  # Llama head_dim
    (7, 1024),  # Qwen3-0.6B hidden size
    (2, 5, 2048),  # Llama 3.2 1B hidden size, batch and sequence dims flattened into rows
    (3, 4100),  # not a multiple of 8: the plain-load path
    (2, 16384),  # a row longer than the bulk path holds in registers: the plain-load path
    (300, 1024),  # several rows per CTA of the row-block kernel's grid
]


def reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm as Hugging Face's Qwen3 and Llama compute it, built on torch's rms_norm."""
    normed = F.rms_norm(x.float(), (x.shape[-1],), eps=eps).to(torch.bfloat16)
    return normed * weight


@pytest.mark.parametrize("shape", SHAPES, ids=str)
def test_matches_torch(device, shape):
    x = random_bf16(*shape, device=device)
    weight = random_bf16(shape[-1], device=device, seed=1)
    assert_close_bf16(svllm_ops.rms_norm(x, weight, EPS), reference(x, weight, EPS))


def test_matches_torch_on_unaligned_rows(device):
    # Starting one element in keeps x contiguous but moves its rows off 16-byte boundaries
    x = random_bf16(4 * 1024 + 1, device=device)[1:].view(4, 1024)
    weight = random_bf16(1024, device=device, seed=1)
    assert_close_bf16(svllm_ops.rms_norm(x, weight, EPS), reference(x, weight, EPS))


@pytest.mark.parametrize(
    "x, weight, message",
    [
        (torch.ones(2, 8), torch.ones(8, dtype=torch.bfloat16), "expected bf16"),
        (torch.ones(2, 8, dtype=torch.bfloat16), torch.ones(4, dtype=torch.bfloat16), "shape"),
        (torch.ones(8, 2, dtype=torch.bfloat16).t(), torch.ones(8, dtype=torch.bfloat16), "contig"),
        (
            torch.ones(2, 8, dtype=torch.bfloat16, device="meta"),
            torch.ones(8, dtype=torch.bfloat16, device="meta"),
            "unsupported device",
        ),
        (
            torch.ones(2, 8, dtype=torch.bfloat16),
            torch.ones(8, dtype=torch.bfloat16, device="meta"),
            "but weight is on",
        ),
    ],
    ids=["fp32", "weight-mismatch", "non-contiguous", "meta-device", "device-mismatch"],
)
def test_rejects_invalid_inputs(x, weight, message):
    with pytest.raises(RuntimeError, match=message):
        svllm_ops.rms_norm(x, weight, EPS)


def test_module_attributes():
    assert svllm_ops.__version__ == "0.1.0"  # the reference's pyproject.toml:3 version
    assert svllm_ops.built_with_cuda is True


# Up to 64 rows per SM (9472 on a B200) the row-block kernel runs; above, the bulk-copy kernels,
# one per row width: both must equal the reference kernel bit for bit. 800 and 1600 leave the
# last pair of a lane's vectors partly or wholly past the row (the paired sums of squares).
BULK_SHAPES = [(10000, 1024), (12000, 128), (10000, 64), (10000, 768), (10000, 2048),
               (10000, 4096), (10000, 96), (10000, 800), (10000, 1600)]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [s for s in SHAPES if s[0]] + [(4096, 1024), (256 * 16, 128),
                                                                  (1000, 768), (50, 4096),
                                                                  (9, 6144), (70, 96)]
                         + BULK_SHAPES, ids=str)
def test_bit_identical_to_reference_cuda_kernel(cuda, shape):
    ref = oracle.reference_module()
    assert ref is not None, "oracle/_ref (the reference's kernels) was not built"
    x = random_bf16(*shape, device=cuda)
    weight = random_bf16(shape[-1], device=cuda, seed=1)
    ours = svllm_ops.rms_norm(x, weight, EPS)
    theirs = ref.rms_norm(x, weight, EPS)  # the reference's CUDA kernel, same GPU
    assert_bf16_within_ulp(ours, theirs, 0, f"rms_norm {shape} vs reference CUDA")


@pytest.mark.gpu
def test_bit_identical_to_reference_cuda_kernel_unaligned(cuda):
    ref = oracle.reference_module()
    x = random_bf16(4 * 1024 + 1, device=cuda)[1:].view(4, 1024)
    weight = random_bf16(1024, device=cuda, seed=1)
    assert torch.equal(svllm_ops.rms_norm(x, weight, EPS), ref.rms_norm(x, weight, EPS))
