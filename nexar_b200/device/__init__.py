"""Device (GPU) side of nexar_b200: symmetric memory and peer-memory collectives."""
from .comm import DeviceCommunicator, GlobalPtr, DeviceHandle  # noqa: F401
