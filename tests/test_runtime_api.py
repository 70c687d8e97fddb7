"""CPU checks of the forge_runtime mirror (forge-runtime/src): the Display
strings of GatherError and PipelineError, and ForgeContext's no-device
error."""
import pytest

from forge_runtime import ForgeContext, GatherError, Pipeline, PipelineError
from forge_sort import DeviceNotFound, GpuExecution


def test_error_display_strings():
    # gather.rs:17-24, pipeline.rs:41-54
    assert str(GatherError.ShaderCompilation("x")) == "shader compilation failed: x"
    assert str(GatherError.GpuExecution("x")) == "GPU execution failed: x"
    assert str(PipelineError.CommandBuffer()) == "failed to create command buffer"
    assert str(PipelineError.Encoder()) == "failed to create compute encoder"
    assert str(PipelineError.GpuExecution("x")) == "GPU execution failed: x"
    assert str(PipelineError.Sort(GpuExecution("x"))) == "sort error: GPU execution failed: x"
    assert isinstance(PipelineError.Sort(GpuExecution("x")), PipelineError)


def test_no_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(DeviceNotFound):
        ForgeContext.new()


def test_pipeline_needs_a_live_context():
    class Closed:
        _stream = 0
    with pytest.raises(PipelineError.CommandBuffer):
        Pipeline(Closed())
