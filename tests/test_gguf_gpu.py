"""GGUF weight source on the GPU: tensors and tensor-parallel shards uploaded from a file
arrive as the exact bytes the file holds, and the kernels read them like any other weights.

The reference maps tensors out of its GGUFFile buffer and uploads raw blocks
(cpp/src/fast_model.cpp:379-470, cpp/src/cuda_kernels.cu:152-156); here the upload streams
the mapped file through pinned staging buffers, a shard's column range of every row or its
row range, straight into device memory."""
from __future__ import annotations

import pytest
import torch

import gguf_files as G
import vibeblade_b200 as vb
from vibeblade_b200 import formats as F
from vibeblade_b200 import tp
from vibeblade_b200.gguf import GGUFFile
from vibeblade_b200.quantize import synthetic_weights

pytestmark = pytest.mark.gpu

# gate (Q4_K, 33 MB: more than one 32 MiB staging chunk), down (Q6_K), a Q8_0 70B-shape
# slice; an F32 bias is added below
SPECS = [("blk.0.ffn_gate.weight", 4096, 14336, F.GGML_TYPE_Q4_K, 1),
         ("blk.0.ffn_down.weight", 14336, 4096, F.GGML_TYPE_Q6_K, 2),
         ("blk.0.attn_q.weight", 8192, 2048, F.GGML_TYPE_Q8_0, 3)]


@pytest.fixture(scope="module")
def model_file(tmp_path_factory, cuda):
    ws = {name: synthetic_weights(K, N, t, seed=s, device=cuda) for name, K, N, t, s in SPECS}
    bias = torch.randn(4096, generator=torch.Generator().manual_seed(4))
    tensors = [G.weight_tensor(name, ws[name].cpu().numpy(), K, N, t) for name, K, N, t, _ in SPECS]
    tensors.append(("blk.0.ffn_down.bias", (4096,), F.GGML_TYPE_F32, bias.numpy().tobytes()))
    kv = [("general.architecture", G.STRING, "llama"), ("llama.embedding_length", G.U32, 4096),
          ("llama.feed_forward_length", G.U32, 14336)]
    path = G.write(tmp_path_factory.mktemp("gguf") / "model.gguf", kv, tensors)
    return path, ws, bias


def test_upload_is_the_file_bytes_and_gemv_reads_it(cuda, model_file):
    path, ws, _ = model_file
    g = torch.Generator(device=cuda).manual_seed(5)
    with GGUFFile(path) as f:
        assert f.meta_int("llama.feed_forward_length") == 14336
        for name, K, N, t, _ in SPECS:
            assert f.matrix_shape(name) == (K, N, t)
            w = f.upload(name, cuda)
            assert w.shape == (K, F.row_bytes(t, N))
            assert torch.equal(w, ws[name].view(K, -1))
            x = torch.randn(4, K, generator=g, device=cuda)
            assert torch.equal(vb.gemv_dequant(x, w, None, K, N, t), vb.gemv_dequant(x, ws[name], None, K, N, t))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_shards_from_the_file(cuda, model_file, world):
    """Column shards of gate and row shards of down, read straight from the file, equal
    vibeblade_b200.tp.shard of the whole uploaded tensor."""
    path, ws, _ = model_file
    with GGUFFile(path) as f:
        for name, kind in (("blk.0.ffn_gate.weight", "column"), ("blk.0.ffn_down.weight", "row")):
            K, N, t = f.matrix_shape(name)
            for r in range(world):
                got = f.upload_shard(name, kind, r, world, cuda)
                assert torch.equal(got, tp.shard(ws[name], K, N, t, kind, r, world))


def test_padded_rows_and_unquantized_bias(cuda, model_file):
    path, ws, bias = model_file
    with GGUFFile(path) as f:
        K, N, t = f.matrix_shape("blk.0.ffn_down.weight")
        rb = F.row_bytes(t, N)
        w = f.upload("blk.0.ffn_down.weight", cuda, rows=(100, 300), cols=(512, 2048), row_bytes=1536)
        src = ws["blk.0.ffn_down.weight"].view(K, rb)[100:300, 2 * 210:8 * 210]
        assert torch.equal(w[:, :6 * 210], src)
        assert torch.count_nonzero(w[:, 6 * 210:]) == 0  # the padding reads as zero
        b = f.upload("blk.0.ffn_down.bias", cuda)
        assert torch.equal(b.view(torch.float32).view(-1).cpu(), bias)
        with pytest.raises(RuntimeError, match="not block-aligned"):
            f.upload("blk.0.ffn_down.weight", cuda, cols=(0, 100))
