"""tpt_spark_b200 -- B200 (sm_100a) engine for tpt-spark's GGUF Llama/Mistral hot path."""
