"""FP32 PyTorch reference of canonical SPAN x2, for parity at full frame sizes (test aid only).

The numpy oracle (oracle/nets.py span_forward, pinned to the reference's interpreter) needs minutes
for one 1920x1080 frame, so the full-size GPU tests compare against this restatement of the same
network in torch FP32 instead (cuDNN / CPU convolutions with TF32 off). tests/test_torch_ref.py pins
it to the numpy oracle on the CPU; the GPU tests pin it again on a crop before they use it."""
from __future__ import annotations

import numpy as np

from oracle import nets


def _fp32_mode():
    import torch
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.deterministic = True


def span_forward(x, p, device="cuda"):
    """nets.span_forward (no quantisation) in torch FP32: x [n,3,h,w] numpy or torch -> numpy
    [n,3,2h,2w], frame by frame to bound device memory."""
    import torch
    import torch.nn.functional as F
    _fp32_mode()
    w = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device) for k, v in p.items()}
    xs = torch.as_tensor(np.asarray(x, np.float32)) if not isinstance(x, torch.Tensor) else x.float()
    outs = []
    with torch.no_grad():
        for i in range(xs.shape[0]):
            xi = xs[i:i + 1].to(device)
            s0 = F.conv2d(xi, w["conv_1.w"], w["conv_1.b"], padding=1)
            xb = s0
            first = last_act = None
            for b in range(nets.SPAN_BLOCKS):
                a1 = F.silu(F.conv2d(xb, w[f"block{b}.c1.w"], w[f"block{b}.c1.b"], padding=1))
                a2 = F.silu(F.conv2d(a1, w[f"block{b}.c2.w"], w[f"block{b}.c2.b"], padding=1))
                c3 = F.conv2d(a2, w[f"block{b}.c3.w"], w[f"block{b}.c3.b"], padding=1)
                xb = (c3 + xb) * (torch.sigmoid(c3) - 0.5)
                if b == 0:
                    first = xb
                if b == nets.SPAN_BLOCKS - 1:
                    last_act = a1
            cat = torch.cat([s0, xb, first, last_act], dim=1)
            fused = F.conv2d(cat, w["conv_cat.w"], w["conv_cat.b"])
            up = F.conv2d(fused, w["upsampler.w"], w["upsampler.b"], padding=1)
            outs.append(F.pixel_shuffle(up, 2).cpu())
            del s0, xb, first, last_act, cat, fused, up
    return torch.cat(outs).numpy()
