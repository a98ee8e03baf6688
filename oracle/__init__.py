"""CPU oracle for the ConvRot W4A4 path. Test infrastructure: not part of the product."""
