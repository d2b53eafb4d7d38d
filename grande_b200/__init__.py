"""omg_b200: the omg decision forward pass (a state prefix plus isolated
question branches in one block-causal pass) as a B200-native engine.

The engine is C++ with hand-written sm_100a CUDA kernels behind the C ABI of
``include/omg_b200.h``; this package loads that library and mirrors the
reference's Rust API (``omg_wgpu::{EngineBuilder, Engine, SavedState}``) on
top of it.
"""
