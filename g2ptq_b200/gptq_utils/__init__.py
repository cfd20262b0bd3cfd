"""Drop-in mirrors of the reference's ``gptq_utils`` quantizer modules."""
