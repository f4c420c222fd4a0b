#define LEO_CUDA_ABI_VERSION 1
struct LeoConfig {
    unsigned int neuron_count;
    unsigned int block_count;
    unsigned int neurons_per_block;
    unsigned int branches_per_neuron;
    unsigned int synapses_per_neuron;
    unsigned int input_fanout;
    unsigned int max_active_per_block;
    unsigned int max_active_global;
    unsigned int context_max_order;
    unsigned int context_embedding_dim;
    unsigned int context_slots_per_order;
    unsigned int context_probe_limit;
    unsigned int context_confidence_observations;
    unsigned int refractory_ticks;
    float branch_decay;
    float membrane_decay;
    float fatigue_decay;
    float fatigue_gain;
    float target_activity;
    float threshold_homeostasis_rate;
    float population_inhibition_rate;
    float population_inhibition_max;
    float adaptation_fast_decay;
    float adaptation_medium_decay;
    float adaptation_slow_decay;
    float adaptation_fast_gain;
    float adaptation_medium_gain;
    float adaptation_slow_gain;
    float membrane_reset_fraction;
    float output_learning_rate;
    float recurrent_learning_rate;
    float inhibitory_learning_rate;
    float eligibility_decay;
    float eligibility_epsilon;
    float surrogate_width;
    float surrogate_gain;
    float max_update;
    float weight_min;
    float weight_max;
    float context_learning_rate;
};
enum LeoPersistentPointerIndex {
    LEO_P_CONFIG = 0,
    LEO_P_THRESHOLD = 1,
    LEO_P_EXCITABILITY = 2,
    LEO_P_NEURON_TYPE = 3,
    LEO_P_RECURRENT_TARGET = 4,
    LEO_P_RECURRENT_BRANCH = 5,
    LEO_P_RECURRENT_DELAY = 6,
    LEO_P_RECURRENT_WEIGHT = 7,
    LEO_P_INPUT_TARGET = 8,
    LEO_P_INPUT_BRANCH = 9,
    LEO_P_INPUT_WEIGHT = 10,
    LEO_P_OUTPUT_WEIGHT = 11,
    LEO_P_OUTPUT_BIAS = 12,
    LEO_P_CONTEXT_KEYS = 13,
    LEO_P_CONTEXT_EMBEDDINGS = 14,
    LEO_P_CONTEXT_OBSERVATIONS = 15,
    LEO_P_CONTEXT_OUTPUT_WEIGHT = 16,
    LEO_P_MEMBRANE = 17,
    LEO_P_ACTIVATION = 18,
    LEO_P_FATIGUE = 19,
    LEO_P_REFRACTORY_UNTIL = 20,
    LEO_P_BRANCHES = 21,
    LEO_P_BRANCH_DELTA = 22,
    LEO_P_BRANCH_LAST_TICK = 23,
    LEO_P_NEURON_LAST_TICK = 24,
    LEO_P_ADAPTATION_FAST = 25,
    LEO_P_ADAPTATION_MEDIUM = 26,
    LEO_P_ADAPTATION_SLOW = 27,
    LEO_P_TOUCHED_EPOCH = 28,
    LEO_P_TOUCHED_LIST = 29,
    LEO_P_TOUCHED_COUNT = 30,
    LEO_P_SELECTED_EPOCH = 31,
    LEO_P_SURROGATE = 32,
    LEO_P_CANDIDATE_ACTIVATION = 33,
    LEO_P_ACTIVE = 34,
    LEO_P_ACTIVE_VALUE = 35,
    LEO_P_ACTIVE_COUNT = 36,
    LEO_P_BLOCK_WINNER_NEURON = 37,
    LEO_P_BLOCK_WINNER_VALUE = 38,
    LEO_P_BLOCK_CUTOFF = 39,
    LEO_P_POPULATION_CUTOFF = 40,
    LEO_P_POPULATION_INHIBITION = 41,
    LEO_P_REC_BRANCH_SENSITIVITY = 42,
    LEO_P_REC_MEMBRANE_SENSITIVITY = 43,
    LEO_P_REC_FATIGUE_SENSITIVITY = 44,
    LEO_P_REC_ADAPTATION_FAST_SENSITIVITY = 45,
    LEO_P_REC_ADAPTATION_MEDIUM_SENSITIVITY = 46,
    LEO_P_REC_ADAPTATION_SLOW_SENSITIVITY = 47,
    LEO_P_REC_ELIGIBILITY = 48,
    LEO_P_REC_LAST_TICK = 49,
    LEO_P_REC_ELIGIBLE_MARK = 50,
    LEO_P_REC_ELIGIBLE_LIST = 51,
    LEO_P_REC_ELIGIBLE_COUNT = 52,
    LEO_P_REC_NEXT_ELIGIBLE_LIST = 53,
    LEO_P_REC_NEXT_ELIGIBLE_COUNT = 54,
    LEO_P_INPUT_BRANCH_SENSITIVITY = 55,
    LEO_P_INPUT_MEMBRANE_SENSITIVITY = 56,
    LEO_P_INPUT_FATIGUE_SENSITIVITY = 57,
    LEO_P_INPUT_ADAPTATION_FAST_SENSITIVITY = 58,
    LEO_P_INPUT_ADAPTATION_MEDIUM_SENSITIVITY = 59,
    LEO_P_INPUT_ADAPTATION_SLOW_SENSITIVITY = 60,
    LEO_P_INPUT_ELIGIBILITY = 61,
    LEO_P_INPUT_LAST_TICK = 62,
    LEO_P_INPUT_ELIGIBLE_MARK = 63,
    LEO_P_INPUT_ELIGIBLE_LIST = 64,
    LEO_P_INPUT_ELIGIBLE_COUNT = 65,
    LEO_P_INPUT_NEXT_ELIGIBLE_LIST = 66,
    LEO_P_INPUT_NEXT_ELIGIBLE_COUNT = 67,
    LEO_P_RING_COUNT = 68,
    LEO_P_RING_SOURCE = 69,
    LEO_P_RING_ACTIVATION = 70,
    LEO_P_RING_WEIGHT = 71,
    LEO_P_CONTEXT_HISTORY = 72,
    LEO_P_CONTEXT_HISTORY_COUNT = 73,
    LEO_P_ACTIVE_CONTEXT_SLOTS = 74,
    LEO_P_ACTIVE_CONTEXT_SCALES = 75,
    LEO_P_ACTIVE_CONTEXT_COUNT = 76,
    LEO_P_CONTEXT_LATENT = 77,
    LEO_P_CONTEXT_GRADIENT = 78,
    LEO_P_NEURAL_LOGITS = 79,
    LEO_P_LOGITS = 80,
    LEO_P_PROBABILITIES = 81,
    LEO_P_ERRORS = 82,
    LEO_P_LEARNING_DESTINATION_EPOCH = 83,
    LEO_P_LEARNING_DESTINATION_LIST = 84,
    LEO_P_LEARNING_DESTINATION_COUNT = 85,
    LEO_P_LEARNING_SIGNAL = 86,
    LEO_P_COUNTERS = 87,
    LEO_P_ERROR_FLAG = 88,
    LEO_P_TRAINING_STEP_RECORDS = 89,
    LEO_P_CHANGED_THRESHOLD_MARKS = 90,
    LEO_P_CHANGED_THRESHOLD_LIST = 91,
    LEO_P_CHANGED_THRESHOLD_COUNT = 92,
    LEO_P_CHANGED_RECURRENT_MARKS = 93,
    LEO_P_CHANGED_RECURRENT_LIST = 94,
    LEO_P_CHANGED_RECURRENT_COUNT = 95,
    LEO_P_CHANGED_INPUT_MARKS = 96,
    LEO_P_CHANGED_INPUT_LIST = 97,
    LEO_P_CHANGED_INPUT_COUNT = 98,
    LEO_P_CHANGED_OUTPUT_MARKS = 99,
    LEO_P_CHANGED_OUTPUT_LIST = 100,
    LEO_P_CHANGED_OUTPUT_COUNT = 101,
    LEO_P_CHANGED_CONTEXT_MARKS = 102,
    LEO_P_CHANGED_CONTEXT_LIST = 103,
    LEO_P_CHANGED_CONTEXT_COUNT = 104,
    LEO_P_POINTER_COUNT = 105
};
enum LeoBatchDeltaPointerIndex {
    LEO_D_THRESHOLD = 0,
    LEO_D_THRESHOLD_MARKS = 1,
    LEO_D_THRESHOLD_LIST = 2,
    LEO_D_THRESHOLD_COUNT = 3,
    LEO_D_RECURRENT = 4,
    LEO_D_RECURRENT_MARKS = 5,
    LEO_D_RECURRENT_LIST = 6,
    LEO_D_RECURRENT_COUNT = 7,
    LEO_D_INPUT = 8,
    LEO_D_INPUT_MARKS = 9,
    LEO_D_INPUT_LIST = 10,
    LEO_D_INPUT_COUNT = 11,
    LEO_D_OUTPUT = 12,
    LEO_D_OUTPUT_MARKS = 13,
    LEO_D_OUTPUT_LIST = 14,
    LEO_D_OUTPUT_COUNT = 15,
    LEO_D_OUTPUT_BIAS = 16,
    LEO_D_CONTEXT_EMBEDDING = 17,
    LEO_D_CONTEXT_MARKS = 18,
    LEO_D_CONTEXT_LIST = 19,
    LEO_D_CONTEXT_COUNT = 20,
    LEO_D_CONTEXT_OBSERVATIONS = 21,
    LEO_D_CONTEXT_OUTPUT = 22,
    LEO_D_POINTER_COUNT = 23
};
static_assert(sizeof(LeoConfig) == 160, "LeoConfig ABI size mismatch");
