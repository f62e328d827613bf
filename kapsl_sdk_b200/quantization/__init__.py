"""kapsl_sdk_b200.quantization"""
