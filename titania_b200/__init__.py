"""titania_b200 — a B200 (sm_100a) device for Titania's Qwen3 model.

The package mirrors the reference's `model` crate interface:

- `B200`: the `Device` trait (model/device.rs) on one GPU, through the C ABI
  of libtitania_b200.so (include/titania_b200.h);
- `Model`, `State`: Model::load / Model::forward (model/model.rs) on the
  fused CUDA-graph decode path;
- `OpModel`, `OpState`: the same forward pass issued one trait call at a time;
- `DeviceSampler`: Sampler::sample (model/sampler.rs) on the device;
- `Config`, `Weights`, `Tensor`, `Sampler`, `BATCH`.

The CUDA library must be built (`python -m titania_b200.build`); there is no
CPU fallback.
"""

from ._lib import DeviceError
from .device import B200, Buffer, Tensor, Weight
from .model import BATCH, BatchState, Config, DeviceSampler, Model, OpModel, OpState, Sampler, State, Weights

__all__ = ["B200", "Buffer", "Tensor", "Weight", "DeviceError", "BATCH", "BatchState", "Config", "DeviceSampler", "Model",
           "OpModel", "OpState", "Sampler", "State", "Weights"]
