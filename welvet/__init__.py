"""welvet: B200-native implementation of welvet.cuda's quantized Dense forward path.

The product is the C-ABI library welvet/cuda_b200/libwelvet_b200.so; `welvet.cuda_b200`
is its Python host binding.
"""
