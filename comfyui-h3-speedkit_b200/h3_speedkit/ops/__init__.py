"""sm_100a CUDA bindings (ctypes over libh3sk_b200.so). No kernel is installed globally."""
