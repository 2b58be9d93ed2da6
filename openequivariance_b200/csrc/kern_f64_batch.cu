#include "kern_table.cuh"
namespace oeqb { OEQB_DEFINE_BATCH_TABLE(double) OEQB_DEFINE_ROW_TABLE(double) OEQB_DEFINE_CW_TABLE(double) }
