"""Generate golden vectors from the reference's own Python emulation.

Runs IST-DASLab/CloverLM's ``src/fake_quartet.py`` (Triton kernels executed
by the Triton interpreter on the CPU, TRITON_INTERPRET=1) on small seeded
inputs and stores inputs and outputs under tests/golden/.  Needs the
reference tree ($CLOVERLM_REF, default: a "reference" directory beside the repository); the committed
.npz files are what the tests read, so the tests never need the reference.

    TRITON_INTERPRET=1 python tests/golden/make_golden.py

Two quirks of running the emulation on a CPU are handled here, not in the
reference: the autotuned launchers need a GPU driver, so the underlying
JIT functions are launched directly with BLOCK_SIZE=2048; and the
interpreter's bf16 tl.dot is wrong, so the EDEN input and Hadamard matrix
are passed as fp32 holding bf16 values (which is exactly what the GPU path
computes: bf16 products accumulated in fp32).
"""
import importlib.util
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")
import numpy as np  # noqa: E402
import torch  # noqa: E402

REF = os.environ.get("CLOVERLM_REF", os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(
    os.path.abspath(__file__)))), "..", "reference"))
HERE = os.path.dirname(os.path.abspath(__file__))


def load_fake():
    spec = importlib.util.spec_from_file_location("fake_quartet", os.path.join(REF, "src", "fake_quartet.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def inputs(seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(128, 512, generator=g)
    idx = torch.randperm(x.numel(), generator=g)[: x.numel() // 1000]
    x.view(-1)[idx] *= 20.0
    t = torch.randn(128, 512, generator=g) / torch.sqrt(torch.randn(128, 512, 3, generator=g).pow(2).mean(-1))
    return x.to(torch.bfloat16), (t / np.sqrt(3.0)).to(torch.bfloat16)


def main():
    fq = load_fake()
    out = {}
    for name, x in zip(("normal_outliers", "student_t"), inputs(0)):
        for four_six in (True, False):
            y = torch.empty_like(x)
            n = x.numel()
            fq._rtn_1x16s_fp4_kernel.fn[(n // 2048,)](
                x_ptr=x, amax_ptr=x.abs().max().float(), output_ptr=y, n_elements=n, scale_override=1.0,
                group_size=16, four_over_six=four_six, BLOCK_SIZE=2048)
            out[f"rtn_{name}_x"] = bits(x)
            out[f"rtn_{name}_{'46' if four_six else 'rne'}_y"] = bits(y)
    # EDEN with a sign-randomized Hadamard: x [128, 512] rotated in 128-groups along rows
    x = inputs(1)[0]
    g = torch.Generator().manual_seed(5)
    H = fq.get_hadamard_matrix(128, torch.float32, "cpu")
    H = (H * (torch.randint(0, 2, (128,), generator=g) * 2 - 1)[None, :]).to(torch.bfloat16)
    so = (17 / 16) * 0.93
    xf = x.float()
    had_t = H.float().T.contiguous()
    amax = (xf.reshape(-1, 128) @ H.float().T).abs().max().float().reshape(1)
    y = torch.empty_like(xf)
    next_amax = torch.zeros(1)
    n = xf.numel()
    fq._eden_1x16s_fp4_kernel.fn[(n // 2048,)](
        x_ptr=xf, hadamard_matrix_ptr=had_t, current_amax_ptr=amax, output_ptr=y, next_amax_ptr=next_amax,
        n_elements=n, hadamard_dim=128, scale_override=so, group_size=16, seed=1234, BLOCK_SIZE=2048)
    out["eden_x"] = bits(x)
    out["eden_h"] = bits(H)
    out["eden_y"] = y.numpy().astype(np.float32)
    out["eden_next_amax"] = next_amax.numpy()
    np.savez_compressed(os.path.join(HERE, "fake_quartet_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "fake_quartet_golden.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    sys.exit(main())
