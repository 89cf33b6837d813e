// tcgen05 int8 matmul (placeholder until the tensor-core path lands)
