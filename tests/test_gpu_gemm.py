"""Grouped GEMM kernels (tcgen05 for bf16/fp16, FFMA for fp32) against a plain PyTorch
fp32 reference of the same op on the same rounded inputs."""
import numpy as np
import pytest
import torch

from util import elementwise_rel_err, max_abs_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from swiftmoe_b200 import kernels
    return kernels


def make_groups(sizes, K_, N, dtype, seed=0, std=0.05):
    g = torch.Generator(device="cpu").manual_seed(seed)
    rows = int(sum(sizes))
    A = torch.randn((max(rows, 1), K_), generator=g).to(dtype)
    B = (torch.randn((len(sizes), N, K_), generator=g) * std).to(dtype)
    B3 = (torch.randn((len(sizes), N, K_), generator=g) * std).to(dtype)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32)
    return A, B, B3, offs, rows


def ref_store(A, B, offs):
    out = torch.zeros((A.shape[0], B.shape[1]), dtype=torch.float64)
    o = offs.tolist()
    for g in range(B.shape[0]):
        out[o[g]:o[g + 1]] = A[o[g]:o[g + 1]].double() @ B[g].double().T
    return out


def ref_swiglu(A, B1, B3, offs):
    g_ = ref_store(A, B1, offs)
    u_ = ref_store(A, B3, offs)
    return torch.nn.functional.silu(g_) * u_


SHAPES = [
    ([128], 64, 256),            # one full tile
    ([1], 64, 256),              # one row
    ([0, 1, 0, 1], 520, 264),    # one token's two experts (decode kernel)
    ([0, 300, 0, 77], 128, 256),  # empty groups, ragged rows
    ([129, 255, 3], 72, 200),    # K % 64 != 0, N % 256 != 0
    ([513, 64, 1000], 256, 512),
    ([37] * 16, 512, 128),       # many small groups
    ([2048, 1536], 1024, 768),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sizes,K_,N", SHAPES)
def test_grouped_store_tc(K, dtype, sizes, K_, N):
    A, B, _, offs, rows = make_groups(sizes, K_, N, dtype, seed=len(sizes) + K_)
    out = K.grouped_gemm(A.cuda(), B.cuda(), offs.cuda())
    ref = ref_store(A, B, offs)[:rows]
    assert elementwise_rel_err(out[:rows].float().cpu().numpy(), ref.numpy()) <= 2e-2
    assert K.read_device_error("cuda") == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sizes,K_,N", SHAPES)
def test_grouped_store_tc_fp32_out(K, dtype, sizes, K_, N):
    A, B, _, offs, rows = make_groups(sizes, K_, N, dtype, seed=7 + K_)
    out = K.grouped_gemm(A.cuda(), B.cuda(), offs.cuda(), out_dtype=torch.float32)
    ref = ref_store(A, B, offs)[:rows].numpy()
    # exact products, fp32 accumulation: error ~ sqrt(K) * 2^-24 * |terms|
    assert max_abs_err(out[:rows].cpu().numpy(), ref) <= 1e-5 * np.sqrt(K_) * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sizes,K_,N", SHAPES)
def test_grouped_swiglu_tc(K, dtype, sizes, K_, N):
    A, B, B3, offs, rows = make_groups(sizes, K_, N, dtype, seed=11 + N)
    out = K.grouped_gemm(A.cuda(), B.cuda(), offs.cuda(), B3=B3.cuda(), epilogue=1)
    ref = ref_swiglu(A, B, B3, offs)[:rows]
    assert elementwise_rel_err(out[:rows].float().cpu().numpy(), ref.numpy()) <= 2e-2


@pytest.mark.parametrize("sizes,K_,N", [([1], 8, 8), ([0, 65, 3], 30, 70), ([200, 130], 512, 256),
                                         ([64] * 9, 96, 64)])
def test_grouped_fp32_simt(K, sizes, K_, N):
    A, B, B3, offs, rows = make_groups(sizes, K_, N, torch.float32, seed=3)
    # fp32 accuracy, 1e-5 absolute at unit output scale: FFMA for K % 4 != 0 or N % 8 != 0,
    # the tf32 tensor cores with split operands (3xTF32) otherwise
    out = K.grouped_gemm(A.cuda(), B.cuda(), offs.cuda())
    ref = ref_store(A, B, offs)[:rows].numpy()
    assert max_abs_err(out[:rows].cpu().numpy(), ref) <= 1e-5 * max(1.0, np.abs(ref).max())
    out = K.grouped_gemm(A.cuda(), B.cuda(), offs.cuda(), B3=B3.cuda(), epilogue=1)
    ref = ref_swiglu(A, B, B3, offs)[:rows].numpy()
    assert max_abs_err(out[:rows].cpu().numpy(), ref) <= 1e-5 * max(1.0, np.abs(ref).max())


def test_grouped_large_mixtral_slice(K):
    """A slice of the Mixtral expert shapes: d=4096 -> 2x14336 gate/up, ragged experts."""
    sizes = [700, 0, 1290, 513]
    A, B, B3, offs, rows = make_groups(sizes, 4096, 1024, torch.bfloat16, seed=5, std=0.02)
    out = K.grouped_gemm(A.cuda(), B.cuda(), offs.cuda(), B3=B3.cuda(), epilogue=1)
    ref = ref_swiglu(A, B, B3, offs)[:rows]
    assert elementwise_rel_err(out[:rows].float().cpu().numpy(), ref.numpy()) <= 2e-2


def test_transpose_batched(K):
    x = torch.randn(3, 70, 45).cuda()
    assert torch.equal(K.transpose_batched(x), x.transpose(1, 2).contiguous())
    xb = x.bfloat16()
    assert torch.equal(K.transpose_batched(xb), xb.transpose(1, 2).contiguous())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_grouped_row_ranges(K, dtype):
    """Groups given as explicit [start, end) row ranges (not contiguous): rows outside
    every range are not written."""
    sizes = [300, 170, 0, 500]
    A, B, B3, offs, rows = make_groups(sizes, 256, 192, dtype, seed=9)
    o = offs.tolist()
    starts = torch.tensor([o[g] + (o[g + 1] - o[g]) // 3 for g in range(4)], dtype=torch.int32)
    ends = torch.tensor([o[g + 1] - (o[g + 1] - o[g]) // 4 for g in range(4)], dtype=torch.int32)
    sentinel = torch.full((rows, 192), 7.0, dtype=dtype, device="cuda")
    out = K.grouped_gemm(A.cuda(), B.cuda(), starts.cuda(), ends=ends.cuda(), out=sentinel)
    ref = ref_store(A, B, offs)
    got = out.float().cpu()
    inside = torch.zeros(rows, dtype=torch.bool)
    for g in range(4):
        inside[starts[g]:ends[g]] = True
    assert (got[~inside] == 7.0).all()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert max_abs_err(got[inside].numpy(), ref[inside].numpy()) <= tol * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("cap", [0, 40])
def test_grouped_gemm_row_addresses(K, dtype, cap):
    """The fused expert-parallel return on one GPU: ep_return_rows turns a receive layout
    (3 source segments x 3 local experts) into one address per expert row, inside a
    buffer where the source regions lie in reverse order; the GEMM with row addresses
    must store exactly the rows of the plain GEMM there, bit for bit, and the rows the
    capacity dropped must become zeros.  Rows outside every region keep their sentinel."""
    ws, El, Kd, N = 3, 3, 256, 192
    rc = torch.tensor([[30, 0, 55], [17, 41, 9], [0, 23, 61]], dtype=torch.int32)
    n_recv = int(rc.sum())
    g = torch.Generator().manual_seed(5)
    xr = torch.randn((n_recv, Kd), generator=g).to(dtype).cuda()
    B = (torch.randn((El, N, Kd), generator=g) * 0.05).to(dtype).cuda()
    rg = K.ep_regroup_plan(rc.cuda(), cap, n_recv)
    xe = K.permute_rows(xr, rg["row_src"], rg["offsets"], rg["rows_cap"])
    y = K.grouped_gemm(xe, B, rg["offsets"])
    per_src = rc.sum(1).tolist()
    starts = np.concatenate([[0], np.cumsum(per_src)]).astype(np.int64)
    pad = 5                                           # rows between regions, never written
    region, at = {}, pad                              # first row of each source region
    for s in reversed(range(ws)):
        region[s] = at
        at += per_src[s] + pad
    buf = torch.full((at, N), 7.0, dtype=dtype, device="cuda")
    rb = N * buf.element_size()
    seg = np.concatenate([starts, [buf.data_ptr() + int(region[s]) * rb for s in range(ws)]]).astype(np.int64)
    row_ptrs = K.ep_return_rows(rg["row_src"], rg["offsets"], rg["recv_dst"], n_recv,
                                torch.from_numpy(seg).cuda(), rb, rg["rows_cap"])
    assert K.grouped_gemm(xe, B, rg["offsets"], row_ptrs=row_ptrs) is None
    got, yc, rd = buf.cpu(), y.cpu(), rg["recv_dst"].cpu().tolist()
    written = torch.zeros(at, dtype=torch.bool)
    for s in range(ws):
        for r in range(int(starts[s]), int(starts[s + 1])):
            row = int(region[s]) + r - int(starts[s])
            written[row] = True
            want = yc[rd[r]] if rd[r] >= 0 else torch.zeros(N, dtype=dtype)
            assert torch.equal(got[row], want), (s, r)
    assert (got[~written] == 7.0).all()
    assert K.read_device_error("cuda") == 0


# Decode-sized batches (at most 2 rows, the warp-per-column kernel) at the shapes that
# matter: the Mixtral gate/up and down projections, K up to 20000, odd K / N, SwiGLU with
# one or two rows per group, a range of columns crossing from one group to the next.
DECODE = [
    ([0, 1, 0, 1], 4096, 2048, 1),     # Mixtral gate/up shape: 2 SwiGLU columns per stage
    ([1, 1], 14336, 1024, 0),          # Mixtral down shape: 1 column per stage, 5 stages
    ([2], 16384, 512, 0),              # two rows of one group, 4 stages
    ([1, 1], 16392, 256, 0),           # 4 stages, K % 256 != 0
    ([0, 1], 64, 1000, 0),             # 4 columns per stage, N % 4 != 0
    ([1, 1], 2056, 300, 1),            # 3 SwiGLU columns per stage, an odd last piece
    ([1, 1], 6144, 700, 0),            # 2 columns per stage
    ([1, 1], 20000, 256, 0),           # 3 stages would fit: warp-per-column kernel
    ([1, 0, 1], 12288, 128, 1),        # SwiGLU, 3 stages would fit: warp-per-column kernel
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sizes,K_,N,epi", DECODE)
def test_decode_gemv(K, dtype, sizes, K_, N, epi):
    A, B, B3, offs, rows = make_groups(sizes, K_, N, dtype, seed=K_ + N, std=0.02)
    Ad, Bd, B3d, od = A.cuda(), B.cuda(), B3.cuda(), offs.cuda()
    if epi:
        out = K.grouped_gemm(Ad, Bd, od, B3=B3d, epilogue=1)
        ref = ref_swiglu(A, B, B3, offs)[:rows]
    else:
        out = K.grouped_gemm(Ad, Bd, od)
        ref = ref_store(A, B, offs)[:rows]
    assert elementwise_rel_err(out[:rows].float().cpu().numpy(), ref.numpy()) <= 2e-2
    again = K.grouped_gemm(Ad, Bd, od, B3=B3d, epilogue=1) if epi else K.grouped_gemm(Ad, Bd, od)
    assert torch.equal(out, again)                     # fixed summation order
    if not epi:
        f32 = K.grouped_gemm(Ad, Bd, od, out_dtype=torch.float32)[:rows].cpu().numpy()
        assert max_abs_err(f32, ref.numpy()) <= 1e-5 * np.sqrt(K_) * max(1.0, float(ref.abs().max()))
    assert K.read_device_error("cuda") == 0


@pytest.mark.parametrize("K_,N", [(14336, 512), (16392, 64)])
def test_decode_gemv_row_addresses(K, K_, N):
    """Two rows stored through row addresses (one null: skipped), bit for bit the rows of
    the plain call."""
    A, B, _, offs, rows = make_groups([1, 0, 1], K_, N, torch.bfloat16, seed=3, std=0.02)
    Ad, Bd, od = A.cuda(), B.cuda(), offs.cuda()
    y = K.grouped_gemm(Ad, Bd, od)
    buf = torch.full((4, N), 7.0, dtype=torch.bfloat16, device="cuda")
    rb = N * 2
    row_ptrs = torch.tensor([buf.data_ptr() + 3 * rb, 0], dtype=torch.int64, device="cuda")
    assert K.grouped_gemm(Ad, Bd, od, row_ptrs=row_ptrs) is None
    got = buf.cpu()
    assert torch.equal(got[3], y[0].cpu())
    assert (got[:3] == 7.0).all()
    assert K.read_device_error("cuda") == 0


# Launches with few tiles (at most half as many as SMs) and long K: the kernel cuts each
# tile's K range into slices on the device and the last slice of a tile to finish sums
# the fp32 partials in slice order.  Ragged N (partly valid tiles), paired [gate | up]
# tiles, fp32 output and output row addresses all go through that path.
SPLIT = [
    ([5, 0, 9], 14336, 4096, 0),      # the Mixtral down projection of a few rows: 32 tiles
    ([7], 8192, 1024, 0),             # 4 tiles, 16 slices
    ([9, 3], 4096, 264, 0),           # N % 256 != 0: the second tile of a group is 8 columns
    ([1, 0, 6], 4096, 2048, 1),       # SwiGLU, 16 paired tiles per group
    ([130], 2048, 200, 1),            # SwiGLU, 2 m-tiles, N % 128 != 0
    ([3, 40], 2048, 512, 3),          # gate and up side by side
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sizes,K_,N,epi", SPLIT)
def test_split_k_few_tiles(K, dtype, sizes, K_, N, epi):
    A, B, B3, offs, rows = make_groups(sizes, K_, N, dtype, seed=K_ + N + epi, std=0.02)
    Ad, Bd, B3d, od = A.cuda(), B.cuda(), B3.cuda(), offs.cuda()

    def run():
        if epi == 1:
            return K.grouped_gemm(Ad, Bd, od, B3=B3d, epilogue=1)
        if epi == 3:                                   # [rows, 2N]: gate | up
            ab = torch.empty((rows, 2 * N), dtype=dtype, device="cuda")
            return K.grouped_gemm(Ad, Bd, od, B3=B3d, epilogue=3, out=ab)
        return K.grouped_gemm(Ad, Bd, od)

    out = run()
    if epi == 1:
        ref = ref_swiglu(A, B, B3, offs)[:rows]
    elif epi == 3:
        ref = torch.cat([ref_store(A, B, offs), ref_store(A, B3, offs)], dim=1)[:rows]
    else:
        ref = ref_store(A, B, offs)[:rows]
    assert elementwise_rel_err(out[:rows].float().cpu().numpy(), ref.numpy()) <= 2e-2
    assert torch.equal(out, run())                     # slices summed in a fixed order
    if epi == 0:
        f32 = K.grouped_gemm(Ad, Bd, od, out_dtype=torch.float32)[:rows].cpu().numpy()
        assert max_abs_err(f32, ref.numpy()) <= 1e-5 * np.sqrt(K_) * max(1.0, float(ref.abs().max()))
    assert K.read_device_error("cuda") == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_split_k_row_addresses(K, dtype):
    """Few tiles with output row addresses: rows land at their addresses (a null
    address skips its row), equal to the rows of the plain call."""
    sizes, K_, N = [4, 0, 3], 14336, 512
    A, B, _, offs, rows = make_groups(sizes, K_, N, dtype, seed=21, std=0.02)
    Ad, Bd, od = A.cuda(), B.cuda(), offs.cuda()
    y = K.grouped_gemm(Ad, Bd, od).cpu()
    buf = torch.full((rows + 2, N), 7.0, dtype=dtype, device="cuda")
    rb = N * buf.element_size()
    dst = [rows + 1 - r if r != 2 else -1 for r in range(rows)]    # reversed, row 2 skipped
    ptrs = torch.tensor([buf.data_ptr() + d * rb if d >= 0 else 0 for d in dst], dtype=torch.int64)
    assert K.grouped_gemm(Ad, Bd, od, row_ptrs=ptrs.cuda()) is None
    got = buf.cpu()
    for r, d in enumerate(dst):
        if d >= 0:
            assert torch.equal(got[d], y[r]), r
    written = {d for d in dst if d >= 0}
    for i in range(rows + 2):
        if i not in written:
            assert (got[i] == 7.0).all(), i
    assert K.read_device_error("cuda") == 0


def test_split_k_interleaved_shapes(K):
    """Split launches of different shapes back to back on one stream: every tile's
    arrival counter is reset by its last slice, so each launch starts from zero."""
    cases = [([3], 14336, 1024), ([2, 2], 4096, 4096), ([5], 14336, 1024)]
    for i, (sizes, K_, N) in enumerate(cases * 2):
        A, B, _, offs, rows = make_groups(sizes, K_, N, torch.bfloat16, seed=i, std=0.02)
        out = K.grouped_gemm(A.cuda(), B.cuda(), offs.cuda())
        ref = ref_store(A, B, offs)[:rows]
        assert elementwise_rel_err(out[:rows].float().cpu().numpy(), ref.numpy()) <= 2e-2, i
    assert K.read_device_error("cuda") == 0


# fp32 grouped GEMMs on the tf32 tensor cores with split operands (3xTF32): the fp32
# layer shapes (d 512, F 2048), ragged and empty groups, a K not a multiple of 32,
# SwiGLU, and launches with few tiles (split-K).  Bar: 1e-5 absolute at unit scale
# against fp64, as for the FFMA kernel; the same call twice is bit-identical.
TF32X3 = [
    ([1000, 0, 1500, 1596], 512, 2048),   # the fp32 layer's gate/up shape (SwiGLU: 2 x 2048)
    ([1000, 0, 1500, 1596], 2048, 512),   # its down projection
    ([37, 300, 5], 100, 264),             # K % 32 != 0, N % 256 != 0
    ([3], 4096, 512),                     # few tiles: split-K slices
    ([700, 300], 14336, 256),             # K > 4096: accumulation chains cut into K slices
]


@pytest.mark.parametrize("sizes,K_,N", TF32X3)
@pytest.mark.parametrize("epi", [0, 1])
def test_fp32_tensor_core_3xtf32(K, sizes, K_, N, epi):
    A, B, B3, offs, rows = make_groups(sizes, K_, N, torch.float32, seed=K_ + N + epi, std=1.0 / np.sqrt(K_))
    Ad, Bd, B3d, od = A.cuda(), B.cuda(), B3.cuda(), offs.cuda()
    run = (lambda: K.grouped_gemm(Ad, Bd, od, B3=B3d, epilogue=1)) if epi else (lambda: K.grouped_gemm(Ad, Bd, od))
    out = run()
    ref = (ref_swiglu(A, B, B3, offs) if epi else ref_store(A, B, offs))[:rows].numpy()
    assert max_abs_err(out[:rows].cpu().numpy(), ref) <= 1e-5 * max(1.0, np.abs(ref).max())
    assert torch.equal(out, run())
    assert K.read_device_error("cuda") == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_grouped_gemm_in_cuda_graph(K, dtype):
    """A grouped GEMM captured into a CUDA graph equals the eager call bit for bit: bf16
    with few tiles (split-K; the capture stream's scratch is allocated during the
    capture), fp32 on the tensor-core path (its scratch grown by an eager call on the
    capture stream first)."""
    sizes, K_, N = ([5, 0, 3], 14336, 1024) if dtype == torch.bfloat16 else ([300, 200], 2048, 512)
    A, B, _, offs, rows = make_groups(sizes, K_, N, dtype, seed=31, std=0.02)
    Ad, Bd, od = A.cuda(), B.cuda(), offs.cuda()
    eager = K.grouped_gemm(Ad, Bd, od)
    out = torch.full_like(eager, 5.0)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    if dtype == torch.float32:                      # the fp32 scratch must exist before capture
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            K.grouped_gemm(Ad, Bd, od, out=out)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        out.fill_(5.0)
    with torch.cuda.graph(g, stream=s):
        K.grouped_gemm(Ad, Bd, od, out=out)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out[:rows], eager[:rows])
    g.replay()                                      # counters reset by the first replay
    torch.cuda.synchronize()
    assert torch.equal(out[:rows], eager[:rows])
    del g
    assert K.read_device_error("cuda") == 0
