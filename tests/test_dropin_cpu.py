"""The onnx-light drop-in (onnx-light_b200/binding) inside onnx-light's own
node runtime, without a GPU: registration through RegisterKernelFn for
Device::kGPU0 + i, the device-keyed dispatch keys RunNode looks up, the
reference's own error for an operator without a GPU kernel
(run_nodes.cc:1597-1600), and no CPU fallback for the registered ones."""
import pytest
import torch

import dropin

pytestmark = pytest.mark.skipif(not __import__("os").path.exists(dropin.HARNESS),
                                reason="oracle/_ref harness not built (needs the reference tree)")


@pytest.fixture(scope="module")
def registered():
    stored = dropin.lib().h_register(2)
    assert stored in (0, 16)  # 8 operators x 2 devices, 0 when already registered
    return True


def key(domain, op, dev):
    import ctypes as C
    buf = C.create_string_buffer(256)
    found = dropin.lib().h_dispatch_key(domain.encode(), op.encode(), dev, buf, 256)
    return found, buf.value.decode()


def test_registration_is_device_keyed(registered):
    for dev in (0, 1):
        for dom, op in (("", "DequantizeLinear"), ("", "MatMulInteger"), ("", "QLinearMatMul"),
                        ("", "Attention"), ("", "RMSNormalization"), ("", "RotaryEmbedding"),
                        ("", "SwiGLU"), ("b200", "DequantizeMatMul")):
            found, k = key(dom, op, dev)
            assert found == 1, k
            assert k == f"{dom or 'ai.onnx'}:{op}:{dev}"
    assert key("", "DequantizeLinear", 2)[0] == 0  # only the devices registered


def test_unregistered_op_on_gpu_raises_the_reference_error(registered):
    with pytest.raises(dropin.NodeError, match="unsupported op_type 'Relu' in domain 'ai.onnx' "
                                              "on device 'GPU0'"):
        dropin.run_node("", "Relu", [(0, 1, (2, 3))], 1, out_bytes=[None])


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_registered_op_resolves_to_the_gpu_kernel_without_cpu_fallback(registered):
    # RunNode picks the GPU kernel, which needs a device: no silent CPU path
    with pytest.raises(dropin.NodeError, match="onnxl_b200 binding"):
        dropin.run_node("", "DequantizeLinear", [(0, 3, (2, 3)), (0, 1, ())], 1, out_bytes=[None])
